"""tcgen05 GEMM (qa_k_gemm) against a plain PyTorch fp32 reference of the same op.

Tolerances: the kernel accumulates in f32 like the reference and rounds once
to the 16-bit output, so the error is the output rounding: max |Δ| / max |ref|
below 2e-3 for f16 and 1e-2 for bf16 outputs; f32 outputs below 1e-4.
"""
import pytest

torch = pytest.importorskip("torch")

from conftest import cuda_ok, pkg  # noqa: E402

pytestmark = pytest.mark.gpu

TOL16 = {torch.float16: 2e-3, torch.bfloat16: 1e-2}


def _lib():
    return pkg()._lib


def _rel(a, b):
    a = a.float()
    b = b.float()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-12)).item()


def _mk(M, N, K, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = (torch.randn(M, K, device="cuda", generator=g) * 0.5).to(dtype)
    B = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(dtype)
    return A, B


@pytest.fixture(autouse=True)
def _need_cuda():
    if not cuda_ok():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 1024, 1024), (1000, 4096, 1024),
                                   (77, 896, 896), (513, 480, 4320), (129, 1024, 3072),
                                   (1, 256, 128), (250, 2688, 896)])
def test_store16(dtype, M, N, K):
    L = _lib()
    A, B = _mk(M, N, K, dtype)
    out = torch.full((M, N), float("nan"), device="cuda", dtype=dtype)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.gemm(A, B, out, status=st)
    torch.cuda.synchronize()
    assert st.item() == 0
    ref = A.float() @ B.float().t()
    assert torch.isfinite(out.float()).all()
    assert _rel(out, ref) < TOL16[dtype]


@pytest.mark.parametrize("bn", [128, 224, 240, 256])
def test_tile_widths(bn):
    L = _lib()
    A, B = _mk(200, 960, 512, torch.float16, seed=bn)
    out = torch.zeros(200, 960, device="cuda", dtype=torch.float16)
    L.gemm(A, B, out, force_bn=bn)
    torch.cuda.synchronize()
    assert _rel(out, A.float() @ B.float().t()) < 2e-3


def test_bias_gelu():
    L = _lib()
    A, B = _mk(333, 3584, 896, torch.float16, seed=3)
    bias = torch.randn(3584, device="cuda") * 0.1
    out = torch.zeros(333, 3584, device="cuda", dtype=torch.float16)
    L.gemm(A, B, out, act=L.ACT_GELU, bias=bias)
    torch.cuda.synchronize()
    ref = torch.nn.functional.gelu(A.float() @ B.float().t() + bias)
    assert _rel(out, ref) < 2e-3


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("m,n,k,bn", [(300, 1024, 2048, 0), (77, 640, 1024, 0), (200, 1024, 1024, 128)])
def test_resid16(dtype, m, n, k, bn):
    """The 16-bit residual epilogue (residual staged through shared memory):
    CTA pairs, a last column tile past N, ragged rows, one-CTA tiles."""
    L = _lib()
    A, B = _mk(m, n, k, dtype, seed=4)
    h = (torch.randn(m, n, device="cuda") * 2).to(dtype)
    ref = (h.float() + A.float() @ B.float().t())
    L.gemm(A, B, h, mode=L.EPI_RESID16, force_bn=bn)
    torch.cuda.synchronize()
    assert _rel(h, ref) < TOL16[dtype]


@pytest.mark.parametrize("m,k,bn", [(250, 3584, 0), (1000, 896, 0), (1000, 896, 128), (700, 896, 224)])
def test_resid32_bias(m, k, bn):
    """The f32 residual epilogue: 64-column blocks with the residual read ahead
    of the accumulator, and the 32-column tail of a 224-wide tile."""
    L = _lib()
    A, B = _mk(m, 896, k, torch.float16, seed=5)
    bias = torch.randn(896, device="cuda") * 0.1
    h = torch.randn(m, 896, device="cuda")
    ref = h + A.float() @ B.float().t() + bias
    L.gemm(A, B, h, mode=L.EPI_RESID32, bias=bias, force_bn=bn)
    torch.cuda.synchronize()
    assert _rel(h, ref) < 1e-4


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_swiglu(dtype):
    """Gate/up rows interleaved in blocks of 128 (half a 256-wide tile)."""
    L = _lib()
    M, I, K = 300, 3072, 1024
    A, _ = _mk(M, 1, K, dtype, seed=6)
    g = torch.Generator(device="cuda").manual_seed(7)
    Wg = (torch.randn(I, K, device="cuda", generator=g) * 0.05).to(dtype)
    Wu = (torch.randn(I, K, device="cuda", generator=g) * 0.05).to(dtype)
    Wp = torch.stack([Wg.view(I // 128, 128, K), Wu.view(I // 128, 128, K)], 1).reshape(2 * I, K)
    out = torch.zeros(M, I, device="cuda", dtype=dtype)
    L.gemm(A, Wp.contiguous(), out, mode=L.EPI_SWIGLU16)
    torch.cuda.synchronize()
    gg = (A.float() @ Wg.float().t()).to(dtype).float()
    uu = (A.float() @ Wu.float().t()).to(dtype).float()
    ref = gg / (1 + torch.exp(-gg)) * uu
    assert _rel(out, ref) < TOL16[dtype]


def test_store32_rowmap_pe():
    L = _lib()
    M, N, K = 260, 896, 7680
    A, B = _mk(M, N, K, torch.float16, seed=8)
    bias = torch.randn(N, device="cuda") * 0.1
    pe = torch.randn(13, N, device="cuda")
    rmap = torch.arange(M, device="cuda", dtype=torch.int32)
    rmap[5::13] = -1
    dst = torch.arange(M, device="cuda")[rmap >= 0]
    rmap[rmap >= 0] = torch.arange(dst.numel(), device="cuda", dtype=torch.int32)
    out = torch.zeros(dst.numel(), N, device="cuda")
    L.gemm(A, B, out, mode=L.EPI_STORE32, bias=bias, row_map=rmap, pe=pe, pe_period=13)
    torch.cuda.synchronize()
    full = A.float() @ B.float().t() + bias + pe[torch.arange(M, device="cuda") % 13]
    ref = full[dst]
    assert _rel(out, ref) < 1e-4


def test_argmax():
    L = _lib()
    M, N, K = 333, 5000, 2048
    A, B = _mk(M, N, K, torch.bfloat16, seed=9)
    logits = torch.zeros(M, N, device="cuda")
    keys = torch.zeros(M, dtype=torch.int64, device="cuda")
    L.gemm(A, B, logits, mode=L.EPI_ARGMAX, keys=keys)
    torch.cuda.synchronize()
    ref = A.float() @ B.float().t()
    assert _rel(logits, ref) < 1e-4
    idx = (0xFFFFFFFF - (keys & 0xFFFFFFFF)).cpu()
    got_from_logits = logits.argmax(1).cpu()
    assert torch.equal(idx, got_from_logits)


def _conv_ref(x_nhwc, w4, bias, time_major):
    """fp32 torch conv2d (3x3, stride 2, pad 1) + bias + erf-GELU, rows in the
    kernel's output order."""
    y = torch.nn.functional.conv2d(x_nhwc.float().permute(0, 3, 1, 2), w4.float(), bias,
                                   stride=2, padding=1)
    y = torch.nn.functional.gelu(y)  # [n, c_out, ho, wo]
    if time_major:
        y = y.permute(0, 3, 2, 1)    # [n, wo, ho, c]
    else:
        y = y.permute(0, 2, 3, 1)    # [n, ho, wo, c]
    return y.reshape(-1, y.shape[-1])


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("n,h,w,c,co,tm", [(3, 64, 50, 480, 480, False), (3, 32, 25, 480, 480, True),
                                          (2, 9, 7, 16, 256, False), (1, 5, 5, 480, 480, True),
                                          (3, 64, 50, 512, 480, False), (3, 32, 25, 512, 480, True),
                                          (1, 5, 5, 512, 480, False)])
def test_implicit_conv(dtype, n, h, w, c, co, tm):
    L = _lib()
    g = torch.Generator(device="cuda").manual_seed(n * h + c)
    x = (torch.randn(n, h, w, c, device="cuda", generator=g) * 0.5).to(dtype)
    w4 = (torch.randn(co, c, 3, 3, device="cuda", generator=g) * 0.05).to(dtype)
    bias = torch.randn(co, device="cuda", generator=g) * 0.1
    wk = w4.permute(0, 2, 3, 1).reshape(co, 9 * c).contiguous()  # k = (kh*3 + kw)*c + ic
    ho, wo = (h - 1) // 2 + 1, (w - 1) // 2 + 1
    out = torch.full((n * ho * wo, co), float("nan"), device="cuda", dtype=dtype)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.conv3x3s2(x, wk, out, time_major=tm, act=L.ACT_GELU, bias=bias, status=st)
    torch.cuda.synchronize()
    assert st.item() == 0
    ref = _conv_ref(x, w4, bias, tm)
    assert torch.isfinite(out.float()).all()
    assert _rel(out, ref) < TOL16[dtype]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_qkv_rope_epilogue(dtype):
    """The fused decoder QKV GEMM (norm_rope_head, src/cpu_decoder.rs:305-321)
    against torch fp32 of the same rounding points: q rows in place, k and v
    appended to shuffled pages of the paged cache, ragged clip lengths."""
    L = _lib()
    nq, nkv, hd, H, page = 16, 8, 128, 1024, 64
    lens = [70, 1, 130, 64, 200]
    g = torch.Generator(device="cuda").manual_seed(7)
    T = sum(lens)
    pages_per = [(n + page - 1) // page for n in lens]
    perm = torch.randperm(sum(pages_per), generator=torch.Generator().manual_seed(3))
    bt = torch.zeros(len(lens), max(pages_per), dtype=torch.int32)
    k = 0
    for c in range(len(lens)):
        bt[c, : pages_per[c]] = perm[k: k + pages_per[c]]
        k += pages_per[c]
    pos = torch.cat([torch.arange(n) for n in lens]).int()
    clip = torch.cat([torch.full((n,), c) for c, n in enumerate(lens)]).int()
    A = (torch.randn(T, H, device="cuda", generator=g)).to(dtype)
    B = (torch.randn((nq + 2 * nkv) * hd, H, device="cuda", generator=g) * 0.03).to(dtype)
    q = torch.full((T, (nq + 2 * nkv) * hd), float("nan"), device="cuda", dtype=dtype)
    kc = torch.zeros(sum(pages_per), nkv, page, hd, device="cuda", dtype=dtype)
    vc = torch.zeros_like(kc)
    ang = torch.arange(512, device="cuda")[:, None] * (1e6 ** (-torch.arange(64, device="cuda") / 64))[None]
    cos_t, sin_t = torch.cos(ang).to(dtype), torch.sin(ang).to(dtype)
    qn = (torch.rand(hd, device="cuda", generator=g) + 0.5).to(dtype).float()
    kn = (torch.rand(hd, device="cuda", generator=g) + 0.5).to(dtype).float()
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    L.gemm_qkv_rope(A, B, q, pos.cuda(), clip.cuda(), bt.cuda(), kc, vc, cos_t, sin_t, qn, kn,
                    1e-6, nq, nkv, status=st)
    torch.cuda.synchronize()
    assert st.item() == 0
    x = (A.float() @ B.float().T).to(dtype).float()
    c = cos_t.float()[pos.long().cuda()]
    s = sin_t.float()[pos.long().cuda()]

    def norm_rope(v, gain):
        inv = 1.0 / torch.sqrt((v * v).mean(-1, keepdim=True) + 1e-6)
        xn = (v * inv) * gain
        a, b = xn[:, :64], xn[:, 64:]
        return torch.cat([a * c - b * s, b * c + a * s], -1).to(dtype).float()

    tol = 1e-2 if dtype == torch.float16 else 3e-2
    for h in range(nq):
        want = norm_rope(x[:, h * hd:(h + 1) * hd], qn)
        got = q[:, h * hd:(h + 1) * hd].float()
        assert torch.isfinite(got).all()
        assert (got - want).abs().max().item() <= tol * want.abs().max().item()
    pg = bt.cuda().long()[clip.long().cuda(), (pos // page).long().cuda()]
    slot = (pos % page).long().cuda()
    for h in range(nkv):
        kw = norm_rope(x[:, (nq + h) * hd:(nq + h + 1) * hd], kn)
        vw = x[:, (nq + nkv + h) * hd:(nq + nkv + h + 1) * hd]
        kg = kc[pg, h, slot].float()
        vg = vc[pg, h, slot].float()
        assert (kg - kw).abs().max().item() <= tol * kw.abs().max().item()
        # v is the rounded GEMM output; torch's fp32 matmul sums in another order
        assert (vg - vw).abs().max().item() <= tol * vw.abs().max().item()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("n,h,w,co", [(3, 128, 100, 480), (1, 9, 7, 480), (2, 16, 13, 64), (2, 9, 7, 40)])
def test_conv1(dtype, n, h, w, co):
    """conv1 (one input channel, 3x3 / stride 2 / pad 1, bias, erf GELU) on the
    tensor cores with split f16 operands (channel counts that are multiples of
    32; 40 takes the CUDA-core kernel), against a float64 torch reference:
    every output within one unit of the 16-bit format's precision."""
    L = _lib()
    g = torch.Generator(device="cuda").manual_seed(11)
    mel = torch.randn(n, h, w, device="cuda", generator=g) * 1.5
    wt = torch.randn(co, 9, device="cuda", generator=g) * 0.3
    bias = torch.randn(co, device="cuda", generator=g) * 0.1
    ho, wo = (h - 1) // 2 + 1, (w - 1) // 2 + 1
    out = torch.full((n * ho * wo, co), float("nan"), device="cuda", dtype=dtype)
    L.conv1(mel, wt, bias, out)
    torch.cuda.synchronize()
    # float64 reference (a float32 cuDNN convolution may run in TF32)
    ref = torch.nn.functional.conv2d(mel[:, None].double(), wt.view(co, 1, 3, 3).double(), bias.double(),
                                     stride=2, padding=1)
    ref = torch.nn.functional.gelu(ref).permute(0, 2, 3, 1).reshape(n * ho * wo, co).float()
    assert torch.isfinite(out.float()).all()
    ulp = 2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7
    err = (out.float() - ref).abs() - ulp * ref.abs()
    assert err.max().item() <= 1e-5
