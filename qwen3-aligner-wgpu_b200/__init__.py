"""B200 (sm_100a) backend for the Qwen3-ForcedAligner alignment path.

The compute lives in libqa_b200.so (CUDA kernels + a C++ host runtime behind
the C ABI of include/qa_b200.h); this package is the Python mirror of the
reference crate's `Aligner` API on top of that ABI, plus the host glue the
reference also keeps on the CPU (word splitting, input building, timestamp
repair) and the seeded synthetic assets the tests and benchmark run on.
"""
from . import _lib  # noqa: F401
from . import audio  # noqa: F401
from . import local_head  # noqa: F401
from . import postprocess  # noqa: F401
from . import rope  # noqa: F401
from . import shard  # noqa: F401
from . import sweep  # noqa: F401
from . import synth  # noqa: F401
from .aligner import Aligner, FORCED_ALIGNER_LANGUAGES  # noqa: F401
from ._lib import QaError  # noqa: F401
