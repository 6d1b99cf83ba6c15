"""The allocation-free RMSNorm backward (jx_rmsnorm_bwd_noalloc), called through the C ABI.

It serves callers that cannot allocate device memory (a runtime bound to the C ABI without a device
allocator, or one held to a fixed budget that must not call cudaMalloc/cudaFree). It runs the same
kernels, on the same grid and in the same reduction order, as the scratch-taking entry point
(jx_rmsnorm_bwd + jx_rmsnorm_dgamma_reduce), so on two calls in a row with different inputs and sizes
its dx and dgamma must equal that entry point's bit for bit; both are also checked against an fp32
autograd F.rms_norm within the per-op tolerance. Sizes beyond its built-in scratch are rejected.
Kept in its own file so it is collected after every other test."""
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 2e-3  # per-op relative tolerance (norm-wise) against the fp32 reference


def _call_noalloc(lib, dy, x, rstd, gamma, dres, dx, dgamma, accumulate):
    rows, cols = x.shape
    lib.call("jx_rmsnorm_bwd_noalloc", dy.data_ptr(), x.data_ptr(), rstd.data_ptr(), gamma.data_ptr(),
             None if dres is None else dres.data_ptr(), dx.data_ptr(), dgamma.data_ptr(), int(accumulate), rows, cols,
             torch.cuda.current_stream().cuda_stream)


def _call_scratch_entry(lib, dy, x, rstd, gamma, dres, dx, dgamma, accumulate):
    rows, cols = x.shape
    nparts = lib.query("jx_rmsnorm_bwd_parts", rows)
    part = torch.empty(nparts * cols, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    lib.call("jx_rmsnorm_bwd", dy.data_ptr(), x.data_ptr(), rstd.data_ptr(), gamma.data_ptr(),
             None if dres is None else dres.data_ptr(), dx.data_ptr(), part.data_ptr(), rows, cols, s)
    lib.call("jx_rmsnorm_dgamma_reduce", part.data_ptr(), nparts, cols, dgamma.data_ptr(), int(accumulate), s)


def _fp32_reference(x, gamma, dy, dres):
    """dx (plus the residual gradient) and dgamma of F.rms_norm computed in fp32 by autograd."""
    xf = x.float().requires_grad_(True)
    gf = gamma.clone().requires_grad_(True)
    y = torch.nn.functional.rms_norm(xf, (x.shape[1],), gf, 1e-5)
    y.backward(dy.float())
    return xf.grad + (dres.float() if dres is not None else 0), gf.grad


# (rows, cols): a full 1024-column case, a small one, and one whose columns need the 4-vector path while
# its rows give fewer blocks (13) than the 296 partial rows the scratch holds.
SHAPES = ((3000, 1024), (777, 256), (100, 1000))


@pytest.mark.parametrize("with_resid", [False, True])
def test_noalloc_matches_scratch_entry_point_twice(with_resid):
    from midstream_llm_b200 import _lib
    torch.cuda.set_device(0)
    for call, (rows, cols) in enumerate(SHAPES):
        g = torch.Generator(device="cuda").manual_seed(10 + call)
        x = torch.randn(rows, cols, device="cuda", generator=g).half()
        dy = torch.randn(rows, cols, device="cuda", generator=g).half()
        dres = torch.randn(rows, cols, device="cuda", generator=g).half() if with_resid else None
        gamma = (1 + 0.1 * torch.randn(cols, device="cuda", generator=g)).float()
        rstd = (x.float().square().mean(-1) + 1e-5).rsqrt().contiguous()
        dx_a, dx_b = torch.empty_like(x), torch.empty_like(x)
        accumulate = call > 0
        init = torch.randn(cols, device="cuda", generator=g) if accumulate else torch.zeros(cols, device="cuda")
        dg_a, dg_b = init.clone(), init.clone()
        _call_noalloc(_lib, dy, x, rstd, gamma, dres, dx_a, dg_a, accumulate)
        _call_scratch_entry(_lib, dy, x, rstd, gamma, dres, dx_b, dg_b, accumulate)
        torch.cuda.synchronize()
        assert torch.equal(dx_a, dx_b), (call, rel_err(dx_a, dx_b))
        assert torch.equal(dg_a, dg_b), (call, rel_err(dg_a, dg_b))
        ref_dx, ref_dg = _fp32_reference(x, gamma, dy, dres)
        assert rel_err(dx_a, ref_dx) < TOL, (call, rel_err(dx_a, ref_dx))
        assert rel_err(dg_a - init, ref_dg) < TOL, (call, rel_err(dg_a - init, ref_dg))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from midstream_llm_b200 import _lib
    x = torch.zeros(16, 2048, device="cuda", dtype=torch.float16)
    with pytest.raises(_lib.JxError, match="exceeds the built-in scratch limit"):
        _call_noalloc(_lib, x, x, torch.ones(16, device="cuda"), torch.ones(2048, device="cuda"), None,
                      torch.empty_like(x), torch.zeros(2048, device="cuda"), False)
