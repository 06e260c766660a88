"""bench.py's algorithmic FLOP count per clip (what `tensor_frac_whole_pass`
divides) against the closed-form count for the default geometry:
F_enc = 4.2080256e9 n_chunks + N_a (13.76256e6 + 18 * 19.267584e6 + 3.44064e6)
        + 18 * sum over windows of 3584 w^2,
F_dec = 880,803,840 L + 114,688 L (L + 1),
F_head = 10,240,000 * 2W."""
import pytest

from conftest import pkg


def closed_form(inp, n_samples):
    frames = n_samples // 160
    chunks = -(-frames // 100)
    na, L, rows = inp.n_audio_tokens, inp.seq_len(), len(inp.timestamp_positions)
    ws = [104] * (na // 104) + ([na % 104] if na % 104 else [])
    f_enc = 4.2080256e9 * chunks + na * (13.76256e6 + 18 * 19.267584e6 + 3.44064e6) \
        + 18 * sum(3584 * w * w for w in ws)
    f_dec = 880_803_840 * L + 114_688 * L * (L + 1)
    return f_enc + f_dec + 10_240_000 * rows


@pytest.mark.parametrize("config,n", [(0, 1), (1, 1), (2, 6), (4, 4)])
def test_model_flops_matches_closed_form(config, n):
    import bench
    qa = pkg()
    cfg = qa.synth.ModelConfig()
    b = qa.synth.InputBuilder(None, n_window=cfg.n_window)
    for clip in qa.synth.workload(config, n_clips=n):
        inp = b.build(qa.synth.split_words(clip.text, clip.language),
                      qa.synth.valid_mel_frames(len(clip.samples)))
        got = bench.model_flops(cfg, inp, len(clip.samples))
        want = closed_form(inp, len(clip.samples))
        assert abs(got - want) <= 1e-9 * want, (config, got, want)
