"""tcgen05 GEMM vs a plain fp32 PyTorch matmul of the same bf16 operands."""
import pytest
import torch

from turbol_b200._native import ops

pytestmark = pytest.mark.gpu


def _ref(A, B, a_mn, b_mn):
    a = A.float().t() if a_mn else A.float()
    b = B.float() if b_mn else B.float().t()
    return a @ b


def _mk(shape, dev, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(shape, generator=g) * 0.5).to(dev, torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 512, 1024), (300, 200, 136), (1000, 384, 520),
                                   (4096, 256, 256), (64, 1536, 1536)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
def test_gemm_layouts(M, N, K, a_mn, b_mn, dev):
    if (a_mn and M % 8) or (b_mn and N % 8):
        pytest.skip("TMA: the contiguous dim of an MN-major operand must be a multiple of 8 (16-byte rows)")
    A = _mk((K, M) if a_mn else (M, K), dev, M + K)
    B = _mk((K, N) if b_mn else (N, K), dev, N + K + 1)
    C = torch.empty(M, N, device=dev, dtype=torch.float32)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops().gemm(A, B, C, a_mn, b_mn, error=err)
    ref = _ref(A, B, a_mn, b_mn)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.allclose(C, ref, atol=2e-2 * (K ** 0.5) / 8, rtol=1e-2), (C - ref).abs().max()


def test_gemm_bf16_out_and_epilogues(dev):
    M, N, K = 777, 512, 256
    A, B = _mk((M, K), dev, 1), _mk((N, K), dev, 2)
    bias = torch.randn(N, device=dev)
    ref = _ref(A, B, False, False)
    o = ops()
    C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    o.gemm(A, B, C, bias=bias, epi=o.EPI_BIAS_TANH)
    assert torch.allclose(C.float(), torch.tanh(ref + bias), atol=2e-2)
    o.gemm(A, B, C, bias=bias, epi=o.EPI_BIAS_SILU)
    assert torch.allclose(C.float(), torch.nn.functional.silu(ref + bias), atol=5e-2, rtol=2e-2)
    H = torch.tanh(torch.randn(M, N, device=dev)).to(torch.bfloat16)
    Cf = torch.empty(M, N, device=dev)
    o.gemm(A, B, Cf, aux=H, epi=o.EPI_TANH_BWD)
    assert torch.allclose(Cf, ref * (1 - H.float() ** 2), atol=2e-2)
    o.gemm(A, B, Cf, aux=H, epi=o.EPI_RESIDUAL)
    assert torch.allclose(Cf, ref + H.float(), atol=2e-2)
    S = torch.empty(M, N // 2, device=dev, dtype=torch.bfloat16)
    o.gemm(A, B, S, epi=o.EPI_SWIGLU)
    exp = torch.nn.functional.silu(ref[:, 0::2]) * ref[:, 1::2]
    assert torch.allclose(S.float(), exp, atol=5e-2, rtol=2e-2)
    o.gemm(A, B, Cf, alpha=0.5)
    assert torch.allclose(Cf, 0.5 * ref, atol=1e-2)


def test_gemm_split_k_and_accumulate(dev):
    # weight-gradient shape: dW[256, 256] = dY^T X over 32768 rows (both MN-major)
    R, N, K = 32768, 256, 256
    dY, X = _mk((R, N), dev, 3), _mk((R, K), dev, 4)
    dW = torch.empty(N, K, device=dev)
    ops().gemm(dY, X, dW, True, True)
    ref = dY.float().t() @ X.float()
    assert torch.allclose(dW, ref, atol=0.5, rtol=1e-2), (dW - ref).abs().max()
    ops().gemm(dY, X, dW, True, True, accumulate=True)
    assert torch.allclose(dW, 2 * ref, atol=1.0, rtol=1e-2)


def test_gemm_splitk_workspace_and_colsum(dev):
    o = ops()
    R, N, K = 32768, 256, 256
    dY, X = _mk((R, N), dev, 5), _mk((R, K), dev, 6)
    ws = torch.zeros(o.gemm_workspace_numel(N, K, R), device=dev)
    assert ws.numel() > 0
    dW = torch.empty(N, K, device=dev)
    o.gemm(dY, X, dW, True, True, workspace=ws)
    ref = dY.float().t() @ X.float()
    assert torch.allclose(dW, ref, atol=0.5, rtol=1e-2)
    # tanh-backward epilogue with fused column sums (a bias gradient)
    M = 3000
    A, B = _mk((M, 64), dev, 7), _mk((64, 256), dev, 8)  # B MN-major [K, N]
    H = torch.tanh(torch.randn(M, 256, device=dev)).to(torch.bfloat16)
    C = torch.empty(M, 256, device=dev, dtype=torch.bfloat16)
    cs = torch.empty(256, device=dev)
    o.gemm(A, B, C, False, True, aux=H, epi=o.EPI_TANH_BWD, colsum=cs)
    exp = (A.float() @ B.float()) * (1 - H.float() ** 2)
    assert torch.allclose(C.float(), exp, atol=3e-2, rtol=2e-2)
    assert torch.allclose(cs, exp.sum(0), atol=0.5, rtol=2e-2)


@pytest.mark.parametrize("epi", ["residual", "tanh_bwd", "bias"])
def test_gemm_splitk_workspace_epilogues(epi, dev):
    # decode-shaped projection: few output tiles, long K -> split-K through the
    # workspace, with the epilogue applied by the reduce pass (bf16 output)
    o = ops()
    M, N, K = 512, 1536, 8960
    A, B = _mk((M, K), dev, 11), _mk((N, K), dev, 12)
    ref = _ref(A, B, False, False)
    H = torch.tanh(torch.randn(M, N, device=dev)).to(torch.bfloat16)
    bias = torch.randn(N, device=dev)
    ws = torch.zeros(o.gemm_workspace_numel(M, N, K), device=dev)
    assert ws.numel() >= 2 * M * N
    C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    # 3 splits: in-kernel fix-up; 7 splits (the automatic count): reduce pass
    for sk in (3, 0):
        if epi == "residual":
            o.gemm(A, B, C, aux=H, epi=o.EPI_RESIDUAL, workspace=ws, split_k=sk)
            exp = ref + H.float()
        elif epi == "tanh_bwd":
            o.gemm(A, B, C, aux=H, epi=o.EPI_TANH_BWD, workspace=ws, split_k=sk)
            exp = ref * (1 - H.float() ** 2)
        else:
            o.gemm(A, B, C, bias=bias, epi=o.EPI_BIAS, workspace=ws, split_k=sk)
            exp = ref + bias
        tol = 2e-2 * exp.abs().max().item()
        assert (C.float() - exp).abs().max().item() < tol, sk


def test_gemm_splitk_inkernel_fixup_accumulate(dev):
    # three splits: the last warp to finish each slice sums the partials in-kernel;
    # fp32 accumulate + alpha + fused column sums, twice in a row (the arrival
    # counters must be left zero by the first call)
    o = ops()
    M, N, K = 300, 200, 4096
    A, B = _mk((M, K), dev, 21), _mk((N, K), dev, 22)
    ref = _ref(A, B, False, False)
    ws = torch.zeros(2 * 1024 * 1024, device=dev)
    C0 = torch.randn(M, N, device=dev)
    C = C0.clone()
    cs = torch.empty(N, device=dev)
    for call in range(2):
        o.gemm(A, B, C, accumulate=True, alpha=0.5, split_k=3, workspace=ws, colsum=cs)
        exp = C0 + 0.5 * ref * (call + 1)
        assert torch.allclose(C, exp, atol=0.05, rtol=1e-2), (call, (C - exp).abs().max())
        assert torch.allclose(cs, 0.5 * ref.sum(0), atol=1.0, rtol=1e-2), call
    assert int(ws[:8192].view(torch.int32).abs().sum()) == 0  # counters back at zero


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_tile_widths(a_mn, b_mn, bn, dev):
    M, N, K = 384, 448, 320
    A = _mk((K, M) if a_mn else (M, K), dev, 31)
    B = _mk((K, N) if b_mn else (N, K), dev, 32)
    C = torch.empty(M, N, device=dev, dtype=torch.float32)
    ops().gemm(A, B, C, a_mn, b_mn, bn=bn)
    ref = _ref(A, B, a_mn, b_mn)
    assert torch.allclose(C, ref, atol=5e-2, rtol=1e-2), (C - ref).abs().max()


def test_gemm_bn64_epilogues(dev):
    # decode-shaped (few rows): the automatic tile width is 64
    o = ops()
    M, N, K = 512, 1536, 1536
    A, B = _mk((M, K), dev, 41), _mk((N, K), dev, 42)
    ref = _ref(A, B, False, False)
    H = torch.randn(M, N, device=dev).to(torch.bfloat16)
    C = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    o.gemm(A, B, C, aux=H, epi=o.EPI_RESIDUAL)
    exp = ref + H.float()
    assert (C.float() - exp).abs().max().item() < 2e-2 * exp.abs().max().item()
    S = torch.empty(M, N // 2, device=dev, dtype=torch.bfloat16)
    o.gemm(A, B, S, epi=o.EPI_SWIGLU, bn=64)
    exp = torch.nn.functional.silu(ref[:, 0::2]) * ref[:, 1::2]
    assert (S.float() - exp).abs().max().item() < 2e-2 * exp.abs().max().item()
    cs = torch.empty(N, device=dev)
    Cf = torch.empty(M, N, device=dev)
    o.gemm(A, B, Cf, bn=64, colsum=cs)
    assert torch.allclose(cs, ref.sum(0), atol=1.0, rtol=1e-2)


@pytest.mark.parametrize("M,N,K,b_mn,bn", [(777, 512, 256, False, 0), (512, 8960, 1536, True, 0),
                                            (300, 272, 320, True, 64), (256, 1024, 512, False, 128)])
def test_gemm_swiglu_save_and_backward_epilogues(M, N, K, b_mn, bn, dev):
    """SwiGLU forward writing the raw gate/up product too (c2), and the
    SwiGLU-backward epilogue (d act -> interleaved d gate, d up), against fp32
    autograd of silu(gate) * up."""
    o = ops()
    A = _mk((M, K), dev, 11)
    B = _mk((K, 2 * N) if b_mn else (2 * N, K), dev, 12)
    ref = _ref(A, B, False, b_mn)                               # [M, 2N] interleaved gate/up
    act = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    gu = torch.empty(M, 2 * N, device=dev, dtype=torch.bfloat16)
    o.gemm(A, B, act, False, b_mn, epi=o.EPI_SWIGLU, c2=gu, bn=bn)
    assert torch.allclose(gu.float(), ref, atol=3e-2, rtol=1e-2), (gu.float() - ref).abs().max()
    g_, u_ = gu.float()[:, 0::2], gu.float()[:, 1::2]
    assert torch.allclose(act.float(), torch.nn.functional.silu(g_) * u_, atol=5e-2, rtol=2e-2)
    # backward: d act = dY . W (the down projection's input gradient), fused into d(gate, up)
    Kd = 384
    dY = _mk((M, Kd), dev, 13)
    Wd = _mk((Kd, N) if b_mn else (N, Kd), dev, 14)       # W stored [K, N] (MN-major) or [N, K]
    d_act = _ref(dY, Wd, False, b_mn)                           # [M, N]
    d_gu = torch.empty(M, 2 * N, device=dev, dtype=torch.bfloat16)
    o.gemm(dY, Wd, d_gu, False, b_mn, aux=gu, epi=o.EPI_SWIGLU_BWD, bn=bn)
    g = g_.clone().requires_grad_()
    u = u_.clone().requires_grad_()
    (torch.nn.functional.silu(g) * u).backward(d_act)
    exp = torch.stack([g.grad, u.grad], -1).reshape(M, 2 * N)
    tol = 3e-2 * max(1.0, float(exp.abs().max()))
    assert torch.allclose(d_gu.float(), exp, atol=tol, rtol=2e-2), (d_gu.float() - exp).abs().max()


@pytest.mark.parametrize("packed", [False, True])
@pytest.mark.parametrize("b_mn", [False, True])
@pytest.mark.parametrize("kg,bn", [(256, 128), (256, 0), (128, 64)])
def test_gemm_block_diagonal_k_range(b_mn, kg, bn, packed, dev):
    """kgroup: output column n reads only the K range of its diagonal block of B.
    B's off-diagonal blocks hold garbage here, so a kernel that still read them
    would not match the fp32 product with the masked (block-diagonal) B.
    packed: B holds only the diagonal blocks, [N, kg] (row r = its block's
    row), inside a wider buffer so that ldb > kg."""
    M, N = 1000, 512
    A = _mk((M, N), dev, 3)
    B = _mk((N, N), dev, 4)
    mask = torch.zeros(N, N, device=dev, dtype=torch.bool)
    for g in range(N // kg):
        mask[g * kg:(g + 1) * kg, g * kg:(g + 1) * kg] = True
    Bm = torch.where(mask, B, torch.zeros_like(B))
    if packed:
        wide = _mk((N, kg + 64), dev, 6)
        for g in range(N // kg):
            wide[g * kg:(g + 1) * kg, :kg] = B[g * kg:(g + 1) * kg, g * kg:(g + 1) * kg]
        B = wide[:, :kg]
    aux = _mk((M, N), dev, 5)
    bias = torch.randn(N, device=dev)
    for epi, kw in ((0, {}), (ops().EPI_BIAS_TANH, {"bias": bias}), (ops().EPI_TANH_BWD, {"aux": aux})):
        C = torch.empty(M, N, device=dev, dtype=torch.bfloat16 if epi else torch.float32)
        ops().gemm(A, B, C, False, b_mn, epi=epi, bn=bn, kgroup=kg, **kw)
        acc = _ref(A, Bm, False, b_mn)
        if epi == ops().EPI_BIAS_TANH:
            acc = torch.tanh(acc + bias)
        elif epi == ops().EPI_TANH_BWD:
            acc = acc * (1 - aux.float() ** 2)
        torch.cuda.synchronize()
        assert torch.allclose(C.float(), acc, atol=3e-2 * (kg ** 0.5) / 8 + 2e-2, rtol=2e-2), (epi, (C.float() - acc).abs().max())


@pytest.mark.parametrize("T,N,K,splits", [(1, 256, 64, 0), (37, 2048, 1536, 0), (256, 1536, 8960, 0),
                                          (300, 384, 520, 3), (200, 1000, 1536, 1), (512, 1536, 1536, 8),
                                          (16, 136, 72, 2)])
@pytest.mark.parametrize("epi", ["none", "bias", "residual", "swiglu"])
def test_gemm_decode_matches_fp32(T, N, K, splits, epi, dev):
    """Weight-stationary decode GEMM (cluster split-K over DSMEM) against the
    fp32 product; odd token counts, a ragged last K block, partial weight
    tiles, several passes of 256 tokens and every epilogue."""
    o = ops()
    X = _mk((T, K), dev, 7)
    W = _mk((N, K), dev, 8)
    acc = X.float() @ W.float().t()
    kw = {}
    code = {"none": o.EPI_NONE, "bias": o.EPI_BIAS, "residual": o.EPI_RESIDUAL, "swiglu": o.EPI_SWIGLU}[epi]
    if epi == "bias":
        kw["bias"] = torch.randn(N, device=dev)
        exp = acc + kw["bias"]
    elif epi == "residual":
        kw["aux"] = _mk((T, N), dev, 9)
        exp = acc + kw["aux"].float()
    elif epi == "swiglu":
        exp = torch.nn.functional.silu(acc[:, 0::2]) * acc[:, 1::2]
    else:
        exp = acc
    C = torch.full((T, N // 2 if epi == "swiglu" else N), float("nan"), device=dev, dtype=torch.bfloat16)
    err = torch.zeros(1, device=dev, dtype=torch.int32)
    o.gemm_decode(X, W, C, epi=code, splits=splits, error=err, **kw)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    tol = 2e-2 * max(1.0, float(exp.abs().max()))
    assert torch.allclose(C.float(), exp, atol=tol, rtol=2e-2), (C.float() - exp).abs().max()


def test_gemm_decode_rejects_misaligned(dev):
    o = ops()
    X = _mk((4, 64), dev, 1)
    W = _mk((12, 64), dev, 2)  # N not a multiple of 8
    C = torch.empty(4, 12, device=dev, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError):
        o.gemm_decode(X, W, C)
