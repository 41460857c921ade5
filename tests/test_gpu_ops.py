"""GPU parity of every single op against the CPU oracle (or exact integer
arithmetic), called through the C ABI on seeded inputs.

Tolerances (written next to each check):
* int8 accumulators and int8 quantisation: bit-exact.
* bf16 outputs: error within a few bf16 ulps of the f32/f64 reference.
* f16 outputs: error within a few f16 ulps (2^-11 relative) of the reference.
* f32 outputs: 1e-4 absolute or tighter.
"""
import math

import numpy as np
import pytest

from oracle import bert as ob
from oracle import quant as oq

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


def _ops():
    from jammi_b200 import ops
    return ops


def _bf16(x, dev):
    return torch.from_numpy(np.asarray(x, dtype=np.float32)).to(dev).to(torch.bfloat16)


# ── linear (tcgen05 bf16) ────────────────────────────────────────────────────

LIN_SHAPES = [  # (M, N, K)
    (1, 768, 768), (37, 96, 32), (128, 256, 64), (300, 2304, 768), (1000, 768, 3072),
    (777, 3072, 768), (64, 512, 768), (5, 16, 48), (256, 128, 1024), (4096, 768, 768),
]


@pytest.mark.parametrize("M,N,K", LIN_SHAPES)
def test_linear_bf16_matches_fp32(dev, M, N, K):
    ops = _ops()
    rng = np.random.default_rng(M * 7 + N + K)
    a = _bf16(rng.standard_normal((M, K)), dev)
    w = _bf16(rng.standard_normal((N, K)) * 0.05, dev)
    bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(dev)
    c = ops.linear(a, w, bias=bias)
    ops.sync()
    ref = a.float() @ w.float().T + bias
    err = (c.float() - ref).abs().max().item()
    # bf16 output rounding: <= 2^-8 relative to the largest |ref| (+ f32 accumulation)
    assert err <= 8e-3 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("epi", ["gelu", "quick_gelu", "residual"])
def test_linear_bf16_epilogues(dev, epi):
    import jammi_b200 as jb
    ops = _ops()
    M, N, K = 333, 768, 768
    rng = np.random.default_rng(5)
    a = _bf16(rng.standard_normal((M, K)), dev)
    w = _bf16(rng.standard_normal((N, K)) * 0.05, dev)
    bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(dev)
    res = _bf16(rng.standard_normal((M, N)), dev)
    z = a.float() @ w.float().T + bias
    if epi == "gelu":
        c = ops.linear(a, w, bias=bias, epilogue=jb.EPI_GELU)
        ref = 0.5 * z * (1 + torch.erf(z / math.sqrt(2)))
    elif epi == "quick_gelu":
        c = ops.linear(a, w, bias=bias, epilogue=jb.EPI_QUICK_GELU)
        ref = z * torch.sigmoid(1.702 * z)
    else:
        c = ops.linear(a, w, bias=bias, residual=res, epilogue=jb.EPI_RESIDUAL)
        ref = z + res.float()
    ops.sync()
    err = (c.float() - ref).abs().max().item()
    assert err <= 8e-3 * ref.abs().max().item() + 1e-3, err


@pytest.mark.parametrize("epi", ["gelu", "quick_gelu"])
def test_tensor_core_activation_accuracy(dev, epi):
    """The tensor-core epilogue's activations against float64: C[m, n] = x_m
    exactly (one non-zero product), so C - act(x) is the activation's own
    error.  GELU uses erf from Abramowitz & Stegun 7.1.28 (|error| <= 3e-7);
    the bar allows that plus the approximate reciprocal / exponential."""
    import jammi_b200 as jb
    ops = _ops()
    x = torch.linspace(-12, 12, 8192).to(torch.bfloat16).float().numpy()
    a = np.zeros((x.size, 64), np.float32)
    a[:, 0] = x
    w = np.zeros((32, 64), np.float32)
    w[:, 0] = 1.0
    e = jb.EPI_GELU if epi == "gelu" else jb.EPI_QUICK_GELU
    c = ops.linear(_bf16(a, dev), _bf16(w, dev), epilogue=e, out_dtype=torch.float32)
    ops.sync()
    xd = x.astype(np.float64)
    if epi == "gelu":
        ref = 0.5 * xd * (1 + np.vectorize(math.erf)(xd / math.sqrt(2)))
    else:
        ref = xd / (1 + np.exp(-1.702 * xd))
    err = np.abs(c.double().cpu().numpy() - ref[:, None])
    assert np.all(err <= 1e-6 * np.maximum(1.0, np.abs(xd))[:, None]), err.max()


def _f16(x, dev):
    return torch.from_numpy(np.asarray(x, dtype=np.float32)).to(dev).to(torch.float16)


@pytest.mark.parametrize("M,N,K", [(1, 768, 768), (300, 2304, 768), (777, 3072, 768), (1000, 768, 3072),
                                   (37, 96, 32), (5, 16, 48)])
def test_linear_f16_matches_fp32(dev, M, N, K):
    """f16 operands on the tcgen05 kernel (kind::f16, A and B both f16), f16
    output: within f16's half ulp (2^-11 of the largest |ref|) plus f32
    accumulation."""
    ops = _ops()
    rng = np.random.default_rng(M * 5 + N + K)
    a = _f16(rng.standard_normal((M, K)), dev)
    w = _f16(rng.standard_normal((N, K)) * 0.05, dev)
    bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(dev)
    c = ops.linear(a, w, bias=bias)
    ops.sync()
    assert c.dtype == torch.float16
    ref = a.double() @ w.double().T + bias.double()
    err = (c.double() - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item() + 1e-4, err


@pytest.mark.parametrize("epi", ["gelu", "residual", "f32_out"])
def test_linear_f16_epilogues(dev, epi):
    import jammi_b200 as jb
    ops = _ops()
    M, N, K = 333, 768, 768
    rng = np.random.default_rng(15)
    a = _f16(rng.standard_normal((M, K)), dev)
    w = _f16(rng.standard_normal((N, K)) * 0.05, dev)
    bias = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(dev)
    res = _f16(rng.standard_normal((M, N)), dev)
    z = a.double() @ w.double().T + bias.double()
    if epi == "gelu":
        c = ops.linear(a, w, bias=bias, epilogue=jb.EPI_GELU)
        ref = 0.5 * z * (1 + torch.erf(z / math.sqrt(2)))
    elif epi == "residual":
        c = ops.linear(a, w, bias=bias, residual=res, epilogue=jb.EPI_RESIDUAL)
        ref = z + res.double()
    else:
        c = ops.linear(a, w, bias=bias, out_dtype=torch.float32)
        ref = z
    ops.sync()
    err = (c.double() - ref).abs().max().item()
    bar = 1e-4 if epi == "f32_out" else 1e-3 * ref.abs().max().item() + 1e-4
    assert err <= bar, err


def test_linear_bf16_f32_output(dev):
    ops = _ops()
    rng = np.random.default_rng(9)
    a = _bf16(rng.standard_normal((200, 768)), dev)
    w = _bf16(rng.standard_normal((512, 768)) * 0.05, dev)
    c = ops.linear(a, w, out_dtype=torch.float32)
    ops.sync()
    ref = a.double() @ w.double().T
    assert (c.double() - ref).abs().max().item() < 1e-4


@pytest.mark.parametrize("M,N,K", [(70, 96, 32), (300, 768, 768), (129, 3072, 384)])
def test_linear_f32_simt(dev, M, N, K):
    ops = _ops()
    rng = np.random.default_rng(M)
    a = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(dev)
    w = torch.from_numpy((rng.standard_normal((N, K)) * 0.05).astype(np.float32)).to(dev)
    b = torch.from_numpy(rng.standard_normal(N).astype(np.float32)).to(dev)
    c = ops.linear(a, w, bias=b)
    ops.sync()
    ref = a.double() @ w.double().T + b.double()
    assert (c.double() - ref).abs().max().item() < 1e-4


# ── int8 (tcgen05 kind::i8): bit-exact accumulators ─────────────────────────

@pytest.mark.parametrize("M,N,K", [(1, 768, 768), (300, 2304, 768), (513, 768, 3072), (129, 4096, 1024),
                                   (77, 96, 32)])
def test_linear_s8_accumulators_bit_exact(dev, M, N, K):
    ops = _ops()
    rng = np.random.default_rng(M + N)
    aq = rng.integers(-127, 128, size=(M, K), dtype=np.int64).astype(np.int8)
    wq = rng.integers(-127, 128, size=(N, K), dtype=np.int64).astype(np.int8)
    aq[0, :] = 127
    wq[0, :] = 127
    wq[1, :] = -127
    a_t = torch.from_numpy(aq).to(dev)
    w_t = torch.from_numpy(wq).to(dev)
    ones_m = torch.ones(M, device=dev)
    ones_n = torch.ones(N, device=dev)
    acc = ops.linear_s8(a_t, ones_m, w_t, ones_n, out_dtype=torch.int32)
    ops.sync()
    ref = oq.gemm_s8_s32(aq, wq)
    got = acc.cpu().numpy()
    assert np.array_equal(got, ref), np.argwhere(got != ref)[:5]
    assert got[0, 0] == K * 127 * 127 and got[0, 1] == -K * 127 * 127


def test_linear_s8_dequant_epilogue(dev):
    import jammi_b200 as jb
    ops = _ops()
    M, N, K = 260, 768, 768
    rng = np.random.default_rng(17)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    xq, xs = oq.quantize_rows(x)
    wq, ws = oq.quantize_rows(w)
    t = lambda v: torch.from_numpy(v).to(dev)
    out = ops.linear_s8(t(xq), t(xs), t(wq), t(ws), bias=t(b), epilogue=jb.EPI_GELU,
                        out_dtype=torch.float32)
    ops.sync()
    z = oq.dequant(oq.gemm_s8_s32(xq, wq), xs, ws, b)
    ref = 0.5 * z * (1 + np.vectorize(math.erf)(z / math.sqrt(2)))
    assert np.abs(out.cpu().numpy() - ref).max() < 1e-4 * np.abs(ref).max() + 1e-5


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_quantize_rows_bit_exact(dev, dtype):
    ops = _ops()
    rng = np.random.default_rng(23)
    x = (rng.standard_normal((513, 3072)) * rng.uniform(0.01, 20, size=(513, 1))).astype(np.float32)
    x[3] = 0
    xt = _bf16(x, dev) if dtype == "bf16" else torch.from_numpy(x).to(dev)
    q, s = ops.quantize_rows(xt)
    ops.sync()
    q_ref, s_ref = oq.quantize_rows(xt.float().cpu().numpy())
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)


def test_gelu_quantize_rows(dev):
    """GELU fused into the per-row quantiser (the int8 FFN2 input): every value
    is looked up in the table of correctly rounded bf16 GELUs, so the int8
    codes and scales equal the oracle's bit for bit.  Rows whose largest value
    reaches 0.5 take the one-pass path (their scale is the GELU of that value);
    the others (scaled down, all negative, all zero) take two passes."""
    ops = _ops()
    from jammi_b200._lib import EPI_GELU
    rng = np.random.default_rng(29)
    x = (rng.standard_normal((777, 3072)) * rng.uniform(0.05, 4, size=(777, 1))).astype(np.float32)
    x[5] = 0
    x[6] = -np.abs(x[6])
    x[7] *= 0.02
    xt = _bf16(x, dev)
    q, s = ops.quantize_rows(xt, activation=EPI_GELU)
    ops.sync()
    xb = xt.double().cpu().numpy()
    assert (xb.max(1) >= 0.5).sum() > 100 and (xb.max(1) < 0.5).sum() > 5   # both paths
    g_bf16 = oq.bf16_round(ob.gelu_erf(xb))
    q_ref, s_ref = oq.quantize_rows(g_bf16)
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().numpy(), s_ref)
    assert s.cpu().numpy()[5] == 0 and not q.cpu().numpy()[5].any()


# ── LayerNorm ───────────────────────────────────────────────────────────────

@pytest.mark.parametrize("dtype,cols,with_res", [
    ("f32", 384, True), ("f32", 32, True), ("bf16", 768, True), ("bf16", 1024, True),
    ("bf16", 64, True), ("bf16", 768, False), ("bf16", 1024, False), ("bf16", 200, False),
    ("f16", 768, True), ("f16", 1024, False), ("f16", 64, False)])
def test_layernorm(dev, dtype, cols, with_res):
    ops = _ops()
    rng = np.random.default_rng(cols)
    R = 1000 if with_res else 4099
    x = (rng.standard_normal((R, cols)) * 3 + 1).astype(np.float32)
    r = rng.standard_normal((R, cols)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, cols).astype(np.float32)
    b = rng.standard_normal(cols).astype(np.float32)
    mk = {"bf16": lambda v: _bf16(v, dev), "f16": lambda v: _f16(v, dev),
          "f32": lambda v: torch.from_numpy(v).to(dev)}[dtype]
    xt, rt = mk(x), mk(r)
    y = ops.layernorm(xt, torch.from_numpy(g).to(dev), torch.from_numpy(b).to(dev), 1e-12,
                      residual=rt if with_res else None)
    ops.sync()
    xin = xt.double().cpu().numpy() + (rt.double().cpu().numpy() if with_res else 0.0)
    ref = ob.layer_norm(xin, g, b, 1e-12)
    err = np.abs(y.double().cpu().numpy() - ref)
    if dtype == "bf16":
        # bf16 output rounding: half an ulp is at most 2^-8 of |y|
        assert np.all(err <= np.abs(ref) * 2.0 ** -8 + 2e-3), err.max()
    elif dtype == "f16":
        # f16 output rounding: half an ulp is at most 2^-11 of |y|
        assert np.all(err <= np.abs(ref) * 2.0 ** -11 + 2e-4), err.max()
    else:
        assert err.max() < 1e-5, err.max()


# ── attention (varlen) ──────────────────────────────────────────────────────

def _attn_ref(qkv, cu, heads, causal=False):
    T, three_h = qkv.shape
    H = three_h // 3
    d = H // heads
    out = np.zeros((T, H))
    for b in range(len(cu) - 1):
        s, e = cu[b], cu[b + 1]
        if e == s:
            continue
        for h in range(heads):
            q = qkv[s:e, h * d:(h + 1) * d]
            k = qkv[s:e, H + h * d:H + (h + 1) * d]
            v = qkv[s:e, 2 * H + h * d:2 * H + (h + 1) * d]
            sc = q @ k.T / math.sqrt(d)
            if causal:  # clip_text.rs:350-362: f32::MIN above the diagonal
                sc = np.where(np.triu(np.ones(sc.shape, dtype=bool), 1), -np.inf, sc)
            out[s:e, h * d:(h + 1) * d] = ob.softmax_last(sc) @ v
    return out


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("lens", [
    [1, 2, 15, 16, 17, 63, 64, 65, 127, 128, 129, 200, 255, 256],
    [300, 17, 257, 256, 1, 512],
])
def test_attention_tc_f16(dev, lens, causal):
    """The tcgen05 kernel with f16 Q, K, V, P and context (kind::f16 with
    both operands f16).  P enters P V as f16 (2^-12 relative, at most ~2e-3
    here against max |V| ~7) and the output is stored as f16 (2^-12 |ref|)."""
    ops = _ops()
    heads, d = 12, 64
    rng = np.random.default_rng(sum(lens) + 11 + (7 if causal else 0))
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = (rng.standard_normal((T + 5, 3 * heads * d)) * 1.5).astype(np.float32)
    qkv[T:] = np.nan
    qt = _f16(qkv, dev)
    ctx = ops.attention(qt.contiguous(), torch.from_numpy(cu).to(dev), heads, max(lens),
                        causal=causal, tma=True)
    ops.sync()
    assert ctx.dtype == torch.float16
    ref = _attn_ref(qt.double().cpu().numpy()[:T], cu, heads, causal=causal)
    got = ctx.double().cpu().numpy()[:T]
    assert np.isfinite(got).all()
    bound = 5e-3 + 5e-4 * np.abs(ref)
    worst = np.abs(got - ref) / bound
    assert worst.max() <= 1.0, (np.abs(got - ref).max(), worst.max())


def test_attention_f16_needs_the_tcgen05_kernel(dev):
    from jammi_b200 import JbError
    ops = _ops()
    qkv = _f16(np.ones((8, 3 * 64)), dev)
    cu = torch.tensor([0, 8], dtype=torch.int32, device=dev)
    ops.set_attention_tcgen05(False)
    try:
        with pytest.raises(JbError):
            ops.attention(qkv, cu, 1, 8, tma=True)
    finally:
        ops.set_attention_tcgen05(True)


@pytest.mark.parametrize("dtype,heads,d,lens", [
    ("bf16", 12, 64, [1, 2, 63, 64, 65, 127, 128, 129, 200, 256]),
    ("bf16", 16, 64, [512, 333, 8, 0, 511]),
    ("bf16", 12, 64, [50] * 7),
    ("f32", 12, 32, [128, 16, 77, 1, 0, 100]),
    ("f32", 2, 16, [16, 9, 1]),
    ("bf16", 4, 8, [5, 5, 5]),
])
def test_attention_varlen(dev, dtype, heads, d, lens):
    ops = _ops()
    rng = np.random.default_rng(sum(lens) + heads)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = (rng.standard_normal((max(T, 1), 3 * heads * d)) * 1.5).astype(np.float32)[:T]
    qt = _bf16(qkv, dev) if dtype == "bf16" else torch.from_numpy(qkv).to(dev)
    if T == 0:
        return
    ctx = ops.attention(qt.contiguous(), torch.from_numpy(cu).to(dev), heads, max(lens))
    ops.sync()
    ref = _attn_ref(qt.double().cpu().numpy(), cu, heads)
    err = np.abs(ctx.double().cpu().numpy() - ref).max()
    tol = 2e-2 if dtype == "bf16" else 1e-5  # bf16: P and V in bf16, outputs |.| < ~3
    assert err < tol, err


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("lens", [
    [1, 2, 15, 16, 17, 63, 64, 65, 127, 128, 129, 200, 255, 256],
    [50] * 7,
    [256, 0, 3, 177],
    [300, 17, 257, 256, 1, 512],
    [700, 129, 1000],
])
@pytest.mark.parametrize("tc", [True, False])
def test_attention_tma_rows(dev, lens, causal, tc):
    """The model forwards' TMA kernels: with tc (the default) every row on the
    tcgen05 kernel (S = QK^T and O = PV as tcgen05.mma, keys in blocks of 128
    with an online softmax); without, the mma.sync one.  The rows after the
    last one hold NaN, as an uninitialised workspace may: keys past a row's end
    must contribute nothing."""
    ops = _ops()
    ops.set_attention_tcgen05(tc)
    heads, d = 12, 64
    rng = np.random.default_rng(sum(lens) + (7 if causal else 0))
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = (rng.standard_normal((T + 5, 3 * heads * d)) * 1.5).astype(np.float32)
    qkv[T:] = np.nan
    qt = _bf16(qkv, dev)
    try:
        ctx = ops.attention(qt.contiguous(), torch.from_numpy(cu).to(dev), heads, max(lens),
                            causal=causal, tma=True)
        ops.sync()
    finally:
        ops.set_attention_tcgen05(True)
    ref = _attn_ref(qt.double().cpu().numpy()[:T], cu, heads, causal=causal)
    got = ctx.double().cpu().numpy()[:T]
    assert np.isfinite(got).all()
    _assert_bf16_ctx(got, ref)


def _assert_bf16_ctx(got, ref):
    """bf16 context against the exact softmax: P enters the P V product as
    bf16 (2^-9 relative: at most 2^-9 of max |V| here, ~0.015) and the output
    is stored as bf16 (half an ulp: 2^-9 |ref|); causal rows' first queries
    see one or two keys, so |ref| reaches max |V| (~7)."""
    bound = 1.5e-2 + 4e-3 * np.abs(ref)
    worst = np.abs(got - ref) / bound
    assert worst.max() <= 1.0, (np.abs(got - ref).max(), worst.max())


def test_attention_tc_rescales_when_a_later_block_dominates(dev):
    """Online softmax across key blocks: keys 128-135 score ~96 and keys
    256-263 ~128 against ~N(0, 4^2) elsewhere, so the second block moves the
    reference maximum by far more than 2^8 (O and the sum rescaled) and the
    third by less (kept, p up to 2^6): both paths against the exact softmax."""
    ops = _ops()
    heads, d = 2, 64
    lens = [300, 260, 140]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    H = heads * d
    rng = np.random.default_rng(5)
    qkv = (rng.standard_normal((T, 3 * H)) * 0.5).astype(np.float32)
    for b, n in enumerate(lens):
        s0 = cu[b]
        qkv[s0:s0 + n, :H] = 1.0                                  # every query = ones
        qkv[s0 + 128:s0 + 136, H:2 * H] = 1.5                     # block 1: scores 96
        if n > 256:
            qkv[s0 + 256:s0 + 264, H:2 * H] = 2.0                 # block 2: scores 128
    qt = _bf16(qkv, dev)
    ctx = ops.attention(qt.contiguous(), torch.from_numpy(cu).to(dev), heads, max(lens), tma=True)
    ops.sync()
    ref = _attn_ref(qt.double().cpu().numpy(), cu, heads)
    got = ctx.double().cpu().numpy()
    assert np.isfinite(got).all()
    _assert_bf16_ctx(got, ref)


@pytest.mark.parametrize("dtype,heads,d,lens", [
    ("bf16", 8, 64, [77, 1, 2, 63, 64, 65, 128, 129, 30]),
    ("bf16", 12, 64, [200, 0, 7]),
    ("f32", 8, 64, [77, 5, 1, 40]),
    ("f32", 4, 16, [24, 7, 2]),
])
def test_attention_causal(dev, dtype, heads, d, lens):
    """The OpenCLIP text mask: query i attends to keys j <= i of its row."""
    ops = _ops()
    rng = np.random.default_rng(sum(lens) + 7 * heads)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = (rng.standard_normal((T, 3 * heads * d)) * 1.5).astype(np.float32)
    qt = _bf16(qkv, dev) if dtype == "bf16" else torch.from_numpy(qkv).to(dev)
    ctx = ops.attention(qt.contiguous(), torch.from_numpy(cu).to(dev), heads, max(lens), causal=True)
    ops.sync()
    ref = _attn_ref(qt.double().cpu().numpy(), cu, heads, causal=True)
    err = np.abs(ctx.double().cpu().numpy() - ref).max()
    tol = 2e-2 if dtype == "bf16" else 1e-5
    assert err < tol, err
    # a row's first query sees only itself: its context is its own V exactly (f32)
    if dtype == "f32":
        H = heads * d
        for b in range(len(lens)):
            if lens[b]:
                r = cu[b]
                np.testing.assert_allclose(ctx[r].cpu().numpy(), qkv[r, 2 * H:], rtol=0, atol=1e-6)


# ── pooling + L2 ────────────────────────────────────────────────────────────

@pytest.mark.parametrize("pooling", ["mean", "cls", "max", "weighted_mean"])
@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
def test_pool_normalize(dev, pooling, dtype):
    ops = _ops()
    rng = np.random.default_rng(3)
    lens = [5, 1, 0, 128, 77]
    H = 768
    S = max(lens)
    hidden = rng.standard_normal((len(lens), S, H)).astype(np.float32)
    mask = (np.arange(S)[None, :] < np.array(lens)[:, None]).astype(np.uint32)
    packed = np.concatenate([hidden[b, :n] for b, n in enumerate(lens)], axis=0)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    pt = {"bf16": lambda: _bf16(packed, dev), "f16": lambda: _f16(packed, dev),
          "f32": lambda: torch.from_numpy(packed).to(dev)}[dtype]()
    out = ops.pool_normalize(pt, torch.from_numpy(cu).to(dev), ob.POOLING_NAMES[pooling])
    ops.sync()
    h_used = np.zeros_like(hidden)
    pk = pt.float().cpu().numpy()
    for b, n in enumerate(lens):
        h_used[b, :n] = pk[cu[b]:cu[b + 1]]
    ref = ob.pool_and_normalize(h_used.astype(np.float32), mask, ob.POOLING_NAMES[pooling])
    got = out.cpu().numpy()
    if pooling == "cls":
        # an all-padding row has no token: the library returns the zero vector
        ref[2] = 0.0
    assert np.all(np.isfinite(got))
    assert np.abs(got - ref).max() < 1e-5
    if pooling in ("mean", "weighted_mean"):
        assert np.all(got[2] == 0)


# ── image preprocessing (image_preprocess.rs:15-75) ──────────────────────────

def test_preprocess_rgb8_bit_exact(dev):
    """White square pad, Catmull-Rom resize and normalisation on the device:
    bit-equal to the f32 restatement for downscales, upscales, the identity
    size, extreme aspect ratios and a 1x1 image."""
    from oracle import image as oimg
    ops = _ops()
    sizes = [(100, 200), (300, 150), (224, 224), (50, 30), (640, 480), (1, 1), (3000, 17), (224, 223)]
    imgs = oimg.random_images(11, sizes)
    mean, std = oimg.OPENAI_CLIP_MEAN, oimg.OPENAI_CLIP_STD
    got = ops.preprocess_rgb8(imgs, 224, mean, std, device=dev).cpu().numpy()
    ref = oimg.preprocess_image_batch(imgs, 224, mean, std)
    assert np.array_equal(got, ref), np.abs(got - ref).max()
    # a small target (the tiny fixtures' 8 x 8) with a large downscale ratio
    got8 = ops.preprocess_rgb8(imgs[:3], 8, (0.5, 0.5, 0.5), (0.25, 0.25, 0.25), device=dev).cpu().numpy()
    assert np.array_equal(got8, oimg.preprocess_image_batch(imgs[:3], 8, (0.5,) * 3, (0.25,) * 3))


def test_bounded_wait_runs_out_and_the_context_stays_usable(dev):
    """Failure detection without a fault: a device-side wait on a flag that
    nothing sets gives up at its limit and reports JB_ERR_TIMEOUT through
    jb_op_sync; a satisfied wait reports nothing, and later ops run."""
    import time
    from jammi_b200 import _lib as L
    ops = _ops()
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    t0 = time.monotonic()
    ops.wait_flag(flag, 1, 200)
    with pytest.raises(L.JbError) as e:
        ops.sync(dev)
    assert e.value.status == L.ERR_TIMEOUT
    assert time.monotonic() - t0 < 10
    flag.fill_(1)
    ops.wait_flag(flag, 1, 200)
    ops.sync(dev)
    x = torch.randn(64, 768, device=dev, dtype=torch.bfloat16)
    q, s = ops.quantize_rows(x)
    torch.cuda.synchronize()
    assert q.shape == (64, 768) and bool(torch.isfinite(s).all())
