// qa_probe_timeout: the failure path of a device pipeline wait, run on
// purpose.  Every tensor-core kernel of the library waits on mbarriers that
// TMA copies or MMA commits complete; each wait is bounded, and one that runs
// out sets the timeout bit of the context's status word, the kernel leaves
// its loops, and the host call returns QA_ERR_TIMEOUT.  This entry point
// launches one CTA whose warp waits (with a caller-given limit) on an
// mbarrier that nothing ever arrives on, which is the state a lost copy or
// commit would leave; it issues no copy and holds no tensor memory, so the
// context stays usable afterwards.
#include <string>

#include "runtime.h"
#include "sm100.cuh"

namespace {

__global__ void wait_probe_kernel(unsigned long long limit_ns, unsigned* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    qa::mbar_init(&bar, 1);  // one arrival would complete phase 0; none comes
    qa::fence_barrier_init();
  }
  __syncthreads();
  const bool ok = __all_sync(0xFFFFFFFFu, qa::mbar_wait_for(&bar, 0, limit_ns));
  if (!ok && threadIdx.x == 0) atomicOr(status, qa::kStatusTimeout);
  __syncthreads();  // nobody still polls the barrier when the CTA exits
}

}  // namespace

extern "C" int qa_probe_timeout(qa_ctx* ctx, int limit_ms) {
  if (!ctx) return QA_ERR_ARG;
  if (limit_ms <= 0 || limit_ms > 10000) {
    ctx->err = "qa_probe_timeout: limit_ms must be in 1..10000";
    return QA_ERR_ARG;
  }
  if (cudaSetDevice(ctx->device) != cudaSuccess) return QA_ERR_CUDA;
  ctx->err.clear();
  cudaStream_t s = ctx->stream;
  if (cudaMemsetAsync(ctx->status.p, 0, 4, s) != cudaSuccess ||
      cudaMemsetAsync(ctx->badflag.p, 0, 4, s) != cudaSuccess) {
    ctx->err = "qa_probe_timeout: cudaMemsetAsync failed";
    return QA_ERR_CUDA;
  }
  wait_probe_kernel<<<1, 32, 0, s>>>(static_cast<unsigned long long>(limit_ms) * 1000000ull,
                                    ctx->status.as<unsigned>());
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    ctx->err = std::string("qa_probe_timeout: launch failed: ") + cudaGetErrorString(e);
    return QA_ERR_CUDA;
  }
  ++ctx->launches;
  const int rc = qa::wait_stream(ctx);
  if (rc) return rc;
  return qa::check_status(ctx);
}
