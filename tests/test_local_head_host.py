"""Host side of the Local Head package: the config.json contract
(HeadFile::validate, src/local_head.rs:661-715), the normalizer and prior
checks, the parameter count (Weights::numel), and the synthetic package
writer — all without a GPU."""
import copy
import json
import os

import numpy as np
import pytest

from conftest import pkg


def test_synthetic_package_round_trips(tmp_path):
    qa = pkg()
    d = qa.synth.write_local_head_dir(str(tmp_path), seed=0)
    assert d == qa.local_head.package_dir(str(tmp_path))
    tensors, mean, std = qa.local_head.load_package(str(tmp_path))
    want, wmean, wstd = qa.synth.random_local_head(0)
    assert set(tensors) == set(want)
    for k in want:
        assert np.array_equal(np.asarray(tensors[k][1]), want[k][1]), k
    assert np.array_equal(mean, wmean) and np.array_equal(std, wstd)
    assert qa.local_head.num_parameters(tensors) == 405264


def test_no_package_is_none(tmp_path):
    assert pkg().local_head.load_package(str(tmp_path)) is None


@pytest.mark.parametrize("path,value", [
    (("schema",), "other"), (("architecture",), "X"), (("context_roles",), ["a"]),
    (("offsets_ms",), [0.0]), (("decoder_temperature",), 1.0),
    (("feature_contract", "n_fft"), 400), (("feature_contract", "center_source"), "argmax"),
    (("model_config", "heads"), 8), (("model_config", "prior_sigma_ms"), 30.0)])
def test_config_contract(path, value):
    qa = pkg()
    cfg = qa.synth.local_head_config_json()
    qa.local_head.validate_config(cfg)
    bad = copy.deepcopy(cfg)
    node = bad
    for k in path[:-1]:
        node = node[k]
    node[path[-1]] = value
    with pytest.raises(ValueError):
        qa.local_head.validate_config(bad)


def test_normalizer_and_prior_checks(tmp_path):
    qa = pkg()
    d = qa.synth.write_local_head_dir(str(tmp_path), seed=1)
    with open(os.path.join(d, "normalizer.json")) as f:
        norm = json.load(f)
    norm["std"][3] = 0.0
    with open(os.path.join(d, "normalizer.json"), "w") as f:
        json.dump(norm, f)
    with pytest.raises(ValueError):
        qa.local_head.load_package(str(tmp_path))
    tensors, _, _ = qa.synth.random_local_head(1)
    tensors["qwen_prior"] = ("F32", np.zeros(13, np.float32))
    with pytest.raises(ValueError):
        qa.local_head.check_prior(tensors)
