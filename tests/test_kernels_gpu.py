"""Per-kernel numerics on the GPU, each against a plain PyTorch fp32 reference
of the same op on the same fp16 inputs. Tolerance: norm-wise relative error
2e-3 (fp16 outputs), 1e-2 for attention / cross-entropy gradients."""
import math

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 2e-3
TOL_ATTN = 1e-2


@pytest.fixture(scope="module")
def ops():
    from midstream_llm_b200 import ops as _ops
    return _ops


@pytest.fixture(params=[0, 1, 2], ids=["auto", "1sm", "2sm"])
def gemm_mode(request, ops):
    """Runs a GEMM test with the library's own kernel choice (the default path), the 1-SM kernel and the
    2-SM (CTA pair) kernel."""
    from midstream_llm_b200 import _lib
    _lib.call("jx_gemm_set_mode", request.param)
    yield request.param
    _lib.call("jx_gemm_set_mode", 0)


def _h(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, device="cuda", generator=g) * scale).half()


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(256, 512, 128), (296, 264, 200), (1024, 3072, 1024)])
def test_gemm_f16_majors(ops, gemm_mode, a_mn, b_mn, M, N, K):
    a = _h(M, K, seed=1)
    b = _h(N, K, seed=2)
    ref = a.float() @ b.float().t()
    A = a.t().contiguous() if a_mn else a
    B = b.t().contiguous() if b_mn else b
    c = ops.gemm_f16(A, B, a_mn_major=a_mn, b_mn_major=b_mn)
    torch.cuda.synchronize()
    assert rel_err(c, ref) < TOL, (a_mn, b_mn, M, N, K, rel_err(c, ref))


def test_gemm_resid(ops, gemm_mode):
    M, N, K = 512, 1024, 1024
    a, b, r = _h(M, K, seed=1), _h(N, K, seed=2), _h(M, N, seed=3)
    c = ops.gemm_f16(a, b, resid=r)
    ref = r.float() + (a.float() @ b.float().t()).half().float()
    assert rel_err(c, ref) < TOL


@pytest.mark.parametrize("M,N,K", [(600, 1056, 704), (1000, 200, 256)])
def test_gemm_resid_ragged(ops, gemm_mode, M, N, K):
    """Residual add with row tiles past M, a last column chunk past N, a residual with its own row
    stride, and in place (the output overwriting the residual)."""
    a, b = _h(M, K, seed=12), _h(N, K, seed=13)
    r = _h(M, N + 40, seed=14)[:, :N]  # leading dimension N + 40
    ref = r.float() + (a.float() @ b.float().t()).half().float()
    assert rel_err(ops.gemm_f16(a, b, resid=r), ref) < TOL
    r2 = r.contiguous()
    assert rel_err(ops.gemm_f16(a, b, resid=r2, out=r2), ref) < TOL


@pytest.mark.parametrize("M", [1, 3, 8])
def test_small_m_products(ops, M):
    """M <= 8 (incremental decoding) takes the weight-streaming path: plain, residual, q/k/v + RoPE at
    arbitrary positions (a one-row slice of the tables) and SwiGLU, with the tiled kernels' rounding."""
    N, K = 1056, 704
    a, b, r = _h(M, K, seed=30), _h(N, K, seed=31), _h(M, N, seed=32)
    assert rel_err(ops.gemm_f16(a, b), a.float() @ b.float().t()) < TOL
    ref = r.float() + (a.float() @ b.float().t()).half().float()
    assert rel_err(ops.gemm_f16(a, b, resid=r), ref) < TOL
    H, hd, T = 3, 64, 512
    d = H * hd
    x, w = _h(M, d, seed=33), _h(3 * d, d, scale=0.05, seed=34)
    cos, sin = _rope_tables(T, hd)
    p0 = 300  # rows of the tables for positions p0 .. p0 + M - 1
    out = ops.gemm_qkv_rope(x, w, d, cos[p0:p0 + M], sin[p0:p0 + M], M, hd)
    lin = (x.float() @ w.float().t()).half().float()
    q, k, v = lin.view(1, M, 3, H, hd).unbind(2)
    cs, sn = cos[p0:p0 + M], sin[p0:p0 + M]
    ref = torch.cat([_rope_ref(q, cs, sn).reshape(M, d), _rope_ref(k, cs, sn).reshape(M, d), v.reshape(M, d)], dim=1)
    assert rel_err(out, ref) < TOL
    F = 320
    wgu = _h(2 * F, d, scale=0.05, seed=35)
    gate, up, act = ops.gemm_swiglu_fwd(x, wgu, F)
    assert rel_err(gate, x.float() @ wgu[:F].float().t()) < TOL
    assert rel_err(up, x.float() @ wgu[F:].float().t()) < TOL
    assert rel_err(act, torch.nn.functional.silu(gate.float()) * up.float()) < TOL


def _rope_tables(T, hd, theta=10000.0):
    inv = theta ** (-torch.arange(0, hd, 2, device="cuda", dtype=torch.float32) / hd)
    ang = torch.arange(T, device="cuda", dtype=torch.float32)[:, None] * inv
    return ang.cos().contiguous(), ang.sin().contiguous()


def _rope_ref(x, cos, sin):
    # x [B, T, H, hd] fp32
    a, b = x.chunk(2, dim=-1)
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    return torch.cat((a * c - b * s, a * s + b * c), dim=-1)


def test_gemm_qkv_rope(ops, gemm_mode):
    B, T, H, hd = 2, 256, 4, 64
    d = H * hd
    x = _h(B * T, d, seed=4)
    w = _h(3 * d, d, scale=0.05, seed=5)
    cos, sin = _rope_tables(T, hd)
    out = ops.gemm_qkv_rope(x, w, d, cos, sin, T, hd)
    lin = (x.float() @ w.float().t()).half().float()
    q, k, v = lin.view(B, T, 3, H, hd).unbind(2)
    ref = torch.cat([_rope_ref(q, cos, sin).reshape(B * T, d), _rope_ref(k, cos, sin).reshape(B * T, d),
                     v.reshape(B * T, d)], dim=1)
    assert rel_err(out, ref) < TOL


@pytest.mark.parametrize("B,T,H", [(3, 256, 5), (5, 96, 4), (3, 200, 4)])
def test_gemm_qkv_rope_shapes(ops, gemm_mode, B, T, H):
    """The 2-SM RoPE epilogue reads a warp's 32 cos / sin rows as TMA boxes when seq_len % 32 == 0 and
    row by row otherwise. Shapes: a tile whose columns straddle the end of q|k (H=5), a partial last
    row tile, seq_len 200."""
    hd = 64
    d = H * hd
    x = _h(B * T, d, seed=40)
    w = _h(3 * d, d, scale=0.05, seed=41)
    cos, sin = _rope_tables(T, hd)
    out = ops.gemm_qkv_rope(x, w, d, cos, sin, T, hd)
    lin = (x.float() @ w.float().t()).half().float()
    q, k, v = lin.view(B, T, 3, H, hd).unbind(2)
    ref = torch.cat([_rope_ref(q, cos, sin).reshape(B * T, d), _rope_ref(k, cos, sin).reshape(B * T, d),
                     v.reshape(B * T, d)], dim=1)
    assert rel_err(out, ref) < TOL


def test_gemm_qkv_rope_table_paths(ops, gemm_mode):
    """One sequence of 768 rows with tables of 769 rows: seq_len 768 (boxes on the 2-SM path) and 769
    (row-by-row reads) rotate every row by the same position, so the outputs are bit-identical.
    Tables that are not 16-byte aligned are rejected on the host."""
    T, H, hd = 768, 5, 64
    d = H * hd
    x = _h(T, d, seed=42)
    w = _h(3 * d, d, scale=0.05, seed=43)
    cos, sin = _rope_tables(T + 1, hd)
    assert torch.equal(ops.gemm_qkv_rope(x, w, d, cos, sin, T, hd), ops.gemm_qkv_rope(x, w, d, cos, sin, T + 1, hd))
    from midstream_llm_b200._lib import JxError
    buf = torch.zeros(cos.numel() + 1, device="cuda", dtype=torch.float32)
    with pytest.raises(JxError, match="16-byte aligned"):
        ops.gemm_qkv_rope(x, w, d, buf[1:].view(T + 1, hd // 2), sin, T + 1, hd)


@pytest.mark.parametrize("M,N,K", [(300, 1000, 256), (1024, 32000, 1024), (64, 2056, 128)])
def test_head_ce_parts(ops, gemm_mode, M, N, K):
    """The tied head with the cross-entropy statistics in its epilogue: its logits equal gemm_f16's bit for
    bit, and lse / loss merged from the per-block statistics match ce_fwd over the stored logits and torch's
    logsumexp (row tiles past M, a last 128-column block past N)."""
    a, b = _h(M, K, seed=50), _h(N, K, scale=0.5, seed=51)
    logits, parts = ops.gemm_f16_ce_parts(a, b)
    assert torch.equal(logits, ops.gemm_f16(a, b))
    g = torch.Generator(device="cuda").manual_seed(52)
    tg = torch.randint(0, N, (M,), device="cuda", generator=g)
    tg[::7] = -100
    lse_ref, loss_ref = ops.ce_fwd(logits, tg)
    lse, loss = ops.ce_fwd_parts(parts, logits, tg)
    assert torch.allclose(lse, lse_ref, rtol=1e-6, atol=1e-5)
    assert torch.allclose(loss, loss_ref, rtol=1e-5, atol=1e-5)
    assert torch.allclose(lse, torch.logsumexp(logits.float(), dim=1), rtol=1e-6, atol=1e-5)


def test_swiglu_fwd_bwd(ops, gemm_mode):
    M, d, F = 512, 256, 688
    x = _h(M, d, seed=6)
    wgu = _h(2 * F, d, scale=0.05, seed=7)
    wd = _h(d, F, scale=0.05, seed=8)
    gate, up, act = ops.gemm_swiglu_fwd(x, wgu, F)
    g_ref = (x.float() @ wgu[:F].float().t())
    u_ref = (x.float() @ wgu[F:].float().t())
    assert rel_err(gate, g_ref) < TOL and rel_err(up, u_ref) < TOL
    act_ref = torch.nn.functional.silu(gate.float()) * up.float()
    assert rel_err(act, act_ref) < TOL
    dy = _h(M, d, seed=9)
    dgu = ops.gemm_swiglu_bwd(dy, wd, gate, up)
    gf = gate.float().requires_grad_(True)
    uf = up.float().requires_grad_(True)
    dact = dy.float() @ wd.float()
    (torch.nn.functional.silu(gf) * uf).backward(dact)
    assert rel_err(dgu[:, :F], gf.grad) < TOL
    assert rel_err(dgu[:, F:], uf.grad) < TOL


def _swiglu_bwd_recipe(dact, gate, up):
    """The fp16-autocast rounding points of silu(gate) * up's backward, in fp32 torch ops:
    d = f16(dact); dup = f16(d * f16(silu(g))); ds = f16(d * u); dgate = f16(ds * s * (1 + g * (1 - s)))."""
    d = dact.half().float()
    g, u = gate.float(), up.float()
    s = torch.sigmoid(g)
    dup = (d * (g * s).half().float()).half()
    ds = (d * u).half().float()
    dgate = (ds * s * (1.0 + g * (1.0 - s))).half()
    return dgate, dup


# (4000, 1024, 2816): the production shape with clipped rows and several tiles per CTA pair (the
# 2-SM epilogue requests gate / up boxes across tile boundaries); (512, 256, 688): a partial last part.
@pytest.mark.parametrize("M,d,F", [(4000, 1024, 2816), (512, 256, 688)])
def test_swiglu_bwd_kernels_agree(ops, M, d, F):
    from midstream_llm_b200 import _lib
    gate, up = _h(M, F, seed=20), _h(M, F, seed=21)
    # Small integers times multiples of 1/64: every partial sum is exact in fp32, so both kernels hold the
    # same accumulators whatever their summation order, and their epilogues must agree bit for bit.
    dy = _h(M, d, scale=1.0, seed=22).float().round().clamp(-2, 2).half()
    wd = (_h(d, F, scale=0.3, seed=23).float() * 64).round().clamp(-64, 64).div(64).half()
    outs = []
    try:
        for mode in (1, 2):
            _lib.call("jx_gemm_set_mode", mode)
            outs.append(ops.gemm_swiglu_bwd(dy, wd, gate, up))
    finally:
        _lib.call("jx_gemm_set_mode", 0)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])  # one formula, bit for bit, in both kernels' epilogues
    dgate, dup = _swiglu_bwd_recipe(dy.float() @ wd.float(), gate, up)
    assert rel_err(outs[1][:, :F], dgate.float()) < TOL
    assert rel_err(outs[1][:, F:], dup.float()) < TOL


def test_swiglu_bwd_repeatable(ops):
    """The pipelined 2-SM epilogue (gate / up requested ahead across tiles, staging reused per part) gives the
    same bits on every run: no part reads a slot or a staging buffer that another request is still filling."""
    M, d, F = 16384, 1024, 2816
    gate, up = _h(M, F, seed=30), _h(M, F, seed=31)
    dy, wd = _h(M, d, seed=32), _h(d, F, scale=0.05, seed=33)
    first = ops.gemm_swiglu_bwd(dy, wd, gate, up)
    out = torch.empty_like(first)
    for _ in range(4):
        out.fill_(float("nan"))
        ops.gemm_swiglu_bwd(dy, wd, gate, up, out=out)
        assert torch.equal(out, first)


# (2048, 2112, 704): the production q/k/v weight gradient, partial tiles in both output dimensions.
@pytest.mark.parametrize("splits,T,N,K", [(1, 2048, 1024, 512), (4, 2048, 1024, 512), (3, 2048, 2112, 704)])
def test_wgrad(ops, gemm_mode, splits, T, N, K):
    dy, x = _h(T, N, seed=10), _h(T, K, seed=11)
    g = torch.randn(N, K, device="cuda")
    g0 = g.clone()
    ops.gemm_wgrad(dy, x, g, accumulate=True, splits=splits)
    ref = g0 + (dy.float().t() @ x.float()).half().float()
    assert rel_err(g, ref) < TOL
    ops.gemm_wgrad(dy, x, g, accumulate=False, splits=splits)
    assert rel_err(g, (dy.float().t() @ x.float())) < TOL


@pytest.mark.parametrize("with_resid", [False, True])
def test_rmsnorm(ops, with_resid):
    rows, cols = 1000, 1024
    x = _h(rows, cols, seed=12)
    r = _h(rows, cols, seed=13) if with_resid else None
    gamma = (1 + 0.1 * torch.randn(cols, device="cuda")).float()
    y, rstd, s = ops.rmsnorm_fwd(x, gamma, 1e-5, resid=r)
    sf = (x.float() + r.float()).half().float() if with_resid else x.float()
    sf.requires_grad_(True)
    gf = gamma.clone().requires_grad_(True)
    yr = torch.nn.functional.rms_norm(sf, (cols,), gf, 1e-5)
    assert rel_err(y, yr) < TOL
    if with_resid:
        assert rel_err(s, sf) < 1e-3
    dy = _h(rows, cols, seed=14)
    dres = _h(rows, cols, seed=15) if with_resid else None
    dx, dg = ops.rmsnorm_bwd(dy, s, rstd, gamma, dresid=dres)
    yr.backward(dy.float())
    ref_dx = sf.grad + (dres.float() if with_resid else 0)
    assert rel_err(dx, ref_dx) < TOL
    assert rel_err(dg, gf.grad) < TOL


@pytest.mark.parametrize("cols,bias,with_resid", [(704, True, True), (1024, False, False), (2112, True, False)])
def test_layernorm(ops, cols, bias, with_resid):
    """LayerNorm as autocast runs it: fp32 layer_norm of the widened fp16 input, fp16 output;
    backward in fp32, input gradient rounded to fp16 and added to the fp16 residual gradient."""
    rows = 1000
    x = _h(rows, cols, seed=40) + 0.5
    gamma = (1 + 0.1 * torch.randn(cols, device="cuda")).float()
    beta = (0.1 * torch.randn(cols, device="cuda")).float() if bias else None
    y, mean, rstd = ops.layernorm_fwd(x, gamma, beta, 1e-5)
    xf = x.float().requires_grad_(True)
    gf = gamma.clone().requires_grad_(True)
    bf = beta.clone().requires_grad_(True) if bias else None
    yr = torch.nn.functional.layer_norm(xf, (cols,), gf, bf, 1e-5)
    assert rel_err(y, yr) < TOL
    assert rel_err(mean, x.float().mean(-1)) < 1e-5
    dy = _h(rows, cols, seed=41)
    dres = _h(rows, cols, seed=42) if with_resid else None
    dbeta = torch.zeros(cols, device="cuda") if bias else None
    dx, dg, db = ops.layernorm_bwd(dy, x, mean, rstd, gamma, dbeta=dbeta, dresid=dres)
    yr.backward(dy.float())
    ref_dx = xf.grad.half().float() + (dres.float() if with_resid else 0)
    assert rel_err(dx, ref_dx) < TOL
    assert rel_err(dg, gf.grad) < TOL
    if bias:
        assert rel_err(db, bf.grad) < TOL


def test_embedding(ops):
    V, d, n = 1000, 256, 4096
    table = torch.randn(V, d, device="cuda")
    ids = torch.randint(0, V, (n,), device="cuda")
    ids[:100] = 7  # a hot row, as Zipf ids produce
    y = ops.embed_fwd(ids, table.half())
    assert torch.equal(y, table.half()[ids])
    dout = _h(n, d, seed=16)
    dt = torch.zeros(V, d, device="cuda")
    ops.embed_bwd(ids, dout, dt)
    ref = torch.zeros(V, d, device="cuda").index_add_(0, ids, dout.float())
    assert rel_err(dt, ref) < 1e-5


def test_cross_entropy(ops):
    rows, V = 512, 32000
    logits = _h(rows, V, scale=3.0, seed=17)
    t = torch.randint(0, V, (rows,), device="cuda")
    t[5] = -100
    lse, row_loss = ops.ce_fwd(logits, t)
    lsc = ops.ce_loss(row_loss, t)
    lf = logits.float().requires_grad_(True)
    ref = torch.nn.functional.cross_entropy(lf, t)
    torch.cuda.synchronize()
    loss = lsc[0] / lsc[1]
    assert abs(float(loss) - float(ref)) / float(ref) < 1e-5
    gl = torch.tensor([65536.0 / 4], device="cuda")
    ref.backward(gl[0])
    d = logits.clone()
    ops.ce_bwd(d, t, lse, gl, lsc[1:2])
    assert rel_err(d, lf.grad) < TOL_ATTN


@pytest.mark.parametrize("bad", [-5, 32000])
def test_cross_entropy_rejects_out_of_range_target(ops, bad):
    """A target outside [0, vocab) that is not ignore_index: torch's cross_entropy refuses it; here the row's
    loss is NaN (so the mean is NaN and the trainer raises), the device status word reads 202, and the
    backward gives that row a zero gradient while the other rows keep theirs."""
    from midstream_llm_b200 import _lib
    rows, V = 64, 32000
    _lib.device_status(clear=True)
    logits = _h(rows, V, scale=3.0, seed=18)
    t = torch.randint(0, V, (rows,), device="cuda")
    t[7] = bad
    lse, row_loss = ops.ce_fwd(logits, t)
    parts = torch.empty(rows, ops.ce_parts_blocks(V), 2, device="cuda")
    # The fused path (statistics from the head GEMM's epilogue) follows the same rule.
    e16 = _h(V, 128, seed=19)
    h16 = _h(rows, 128, seed=20)
    lg2, _ = ops.gemm_f16_ce_parts(h16, e16, parts=parts)
    _, row_loss2 = ops.ce_fwd_parts(parts, lg2, t)
    lsc = ops.ce_loss(row_loss, t)
    torch.cuda.synchronize()
    assert torch.isnan(row_loss[7]) and torch.isnan(row_loss2[7]) and torch.isnan(lsc[2])
    others = torch.arange(rows, device="cuda") != 7
    assert torch.isfinite(row_loss[others]).all() and torch.isfinite(row_loss2[others]).all()
    assert _lib.device_status(clear=True) == 202
    d = logits.clone()
    ops.ce_bwd(d, t, lse, torch.tensor([1.0], device="cuda"), torch.tensor([float(rows - 1)], device="cuda"))
    torch.cuda.synchronize()
    assert torch.count_nonzero(d[7]) == 0 and torch.count_nonzero(d[8]) > 0
    assert _lib.device_status(clear=True) == 0


def _attn_ref(q, k, v):
    # q,k,v [B,H,T,D] fp32
    T = q.shape[2]
    s = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
    s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    return s.softmax(-1) @ v


# (8, 1024, 16) and (1, 4096, 16) have more work items (query-tile pairs / key blocks
# of each head) than the GPU has SMs, so each persistent CTA runs several of them.
@pytest.mark.parametrize("B,T,H", [(2, 256, 4), (1, 1024, 2), (8, 1024, 16), (1, 4096, 16)])
def test_attention(ops, B, T, H):
    D = 64
    d = H * D
    qkv = _h(B * T, 3 * d, seed=18)
    o, lse = ops.attn_fwd(qkv, B, T, H, D)
    q, k, v = [t.float().view(B, T, H, D).transpose(1, 2).requires_grad_(True)
               for t in qkv.view(B * T, 3, d).unbind(1)]
    ref = _attn_ref(q, k, v)
    assert rel_err(o, ref.transpose(1, 2).reshape(B * T, d)) < TOL
    do = _h(B * T, d, seed=19)
    ref.backward(do.float().view(B, T, H, D).transpose(1, 2))
    dqkv = ops.attn_bwd(qkv, o, do, lse, B, T, H, D)
    dq, dk, dv = [t.view(B, T, H, D).transpose(1, 2) for t in dqkv.view(B * T, 3, d).unbind(1)]
    assert rel_err(dv, v.grad) < TOL_ATTN
    assert rel_err(dk, k.grad) < TOL_ATTN
    assert rel_err(dq, q.grad) < TOL_ATTN


def test_attention_rope_bwd(ops):
    B, T, H, D = 1, 256, 2, 64
    d = H * D
    qkv = _h(B * T, 3 * d, seed=20)
    cos, sin = _rope_tables(T, D)
    o, lse = ops.attn_fwd(qkv, B, T, H, D)
    do = _h(B * T, d, seed=21)
    plain = ops.attn_bwd(qkv, o, do, lse, B, T, H, D)
    rot = ops.attn_bwd(qkv, o, do, lse, B, T, H, D, cos=cos, sin=sin)
    # inverse rotation of the plain q/k gradients
    for part in range(2):
        g = plain[:, part * d:(part + 1) * d].float().view(B, T, H, D)
        g1, g2 = g.chunk(2, dim=-1)
        c, s = cos[None, :, None, :], sin[None, :, None, :]
        ref = torch.cat((g1 * c + g2 * s, g2 * c - g1 * s), dim=-1).reshape(B * T, d)
        assert rel_err(rot[:, part * d:(part + 1) * d], ref) < TOL
    assert torch.equal(rot[:, 2 * d:], plain[:, 2 * d:])


@pytest.mark.parametrize("grad_f16", [False, True])
def test_adamw_matches_torch(ops, grad_f16):
    n = 100_003
    p = torch.randn(n, device="cuda") * 0.02
    g32 = torch.randn(n, device="cuda") * 1e-3 * 1024
    g = g32.half() if grad_f16 else g32
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    tp = p.clone().requires_grad_(True)
    opt = torch.optim.AdamW([tp], lr=3e-4, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1, fused=True)
    inv = torch.tensor([1 / 1024.0], device="cuda")
    partial = torch.empty(ops.grad_stats_parts(n), device="cuda")
    found = torch.zeros(1, device="cuda")
    nparts = ops.grad_stats(g, inv, partial, found)
    fin = torch.empty(2, device="cuda")
    ops.grad_finalize(partial, nparts, 1.0, fin)
    gu = g.float() * inv
    total = gu.norm()
    coef = torch.clamp(1.0 / (total + 1e-6), max=1.0)
    torch.cuda.synchronize()
    assert abs(float(fin[0]) - float(total)) / float(total) < 1e-5
    p16 = torch.empty(n, device="cuda", dtype=torch.float16)
    state = torch.zeros(4, device="cuda")
    for step in (1, 2):
        ops.adamw_step(p, g, m, v, p16, inv, fin[1:2], found, state, 3e-4, 0.9, 0.95, 1e-5, 0.1)
        tp.grad = gu * coef
        opt.step()
    torch.cuda.synchronize()
    assert torch.allclose(p, tp.detach(), rtol=1e-6, atol=1e-9)
    assert torch.equal(p16, p.half())
    assert float(state[0]) == 2.0


def test_adamw_skips_on_inf(ops):
    n = 4096
    p = torch.randn(n, device="cuda")
    g = torch.randn(n, device="cuda")
    g[17] = float("inf")
    m, v = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
    inv = torch.ones(1, device="cuda")
    partial = torch.empty(ops.grad_stats_parts(n), device="cuda")
    found = torch.zeros(1, device="cuda")
    ops.grad_stats(g, inv, partial, found)
    p0 = p.clone()
    state = torch.zeros(4, device="cuda")
    ops.adamw_step(p, g, m, v, None, inv, None, found, state, 1e-3, 0.9, 0.95, 1e-5, 0.1)
    torch.cuda.synchronize()
    assert float(found) == 1.0
    assert torch.equal(p, p0) and not m.any()
    assert float(state[0]) == 0.0


def test_scaler_update(ops):
    scale = torch.tensor([65536.0], device="cuda")
    tracker = torch.zeros(1, device="cuda", dtype=torch.int32)
    found = torch.zeros(1, device="cuda")
    ops.scaler_update(scale, tracker, found, interval=2)
    ops.scaler_update(scale, tracker, found, interval=2)
    torch.cuda.synchronize()
    assert float(scale) == 131072.0 and int(tracker) == 0
    found.fill_(1.0)
    ops.scaler_update(scale, tracker, found, interval=2)
    torch.cuda.synchronize()
    assert float(scale) == 65536.0
