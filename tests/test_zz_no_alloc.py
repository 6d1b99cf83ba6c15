"""The allocation-free RMSNorm backward (jx_rmsnorm_bwd_noalloc), for callers that
cannot allocate device memory, called through the C ABI: its dx and dgamma match
the scratch-taking entry point (jx_rmsnorm_bwd + jx_rmsnorm_dgamma_reduce) on two
calls in a row with different inputs, and sizes beyond its built-in scratch are
rejected. Kept in its own file so it is collected after every other test."""
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _call_noalloc(lib, dy, x, rstd, gamma, dres, dx, dgamma, accumulate):
    rows, cols = x.shape
    lib.call("jx_rmsnorm_bwd_noalloc", dy.data_ptr(), x.data_ptr(), rstd.data_ptr(), gamma.data_ptr(),
             None if dres is None else dres.data_ptr(), dx.data_ptr(), dgamma.data_ptr(), int(accumulate), rows, cols,
             torch.cuda.current_stream().cuda_stream)


def _call_reference_entry(lib, dy, x, rstd, gamma, dres, dx, dgamma, accumulate):
    rows, cols = x.shape
    nparts = lib.query("jx_rmsnorm_bwd_parts", rows)
    part = torch.empty(nparts * cols, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    lib.call("jx_rmsnorm_bwd", dy.data_ptr(), x.data_ptr(), rstd.data_ptr(), gamma.data_ptr(),
             None if dres is None else dres.data_ptr(), dx.data_ptr(), part.data_ptr(), rows, cols, s)
    lib.call("jx_rmsnorm_dgamma_reduce", part.data_ptr(), nparts, cols, dgamma.data_ptr(), int(accumulate), s)


@pytest.mark.parametrize("with_resid", [False, True])
def test_noalloc_matches_scratch_entry_point_twice(with_resid):
    from midstream_llm_b200 import _lib
    torch.cuda.set_device(0)
    for call, (rows, cols) in enumerate(((3000, 1024), (777, 256))):
        g = torch.Generator(device="cuda").manual_seed(10 + call)
        x = torch.randn(rows, cols, device="cuda", generator=g).half()
        dy = torch.randn(rows, cols, device="cuda", generator=g).half()
        dres = torch.randn(rows, cols, device="cuda", generator=g).half() if with_resid else None
        gamma = (1 + 0.1 * torch.randn(cols, device="cuda", generator=g)).float()
        rstd = (x.float().square().mean(-1) + 1e-5).rsqrt().contiguous()
        dx_a, dx_b = torch.empty_like(x), torch.empty_like(x)
        init = torch.randn(cols, device="cuda", generator=g)
        dg_a, dg_b = init.clone(), init.clone()
        _call_noalloc(_lib, dy, x, rstd, gamma, dres, dx_a, dg_a, accumulate=(call == 1))
        _call_reference_entry(_lib, dy, x, rstd, gamma, dres, dx_b, dg_b, accumulate=(call == 1))
        torch.cuda.synchronize()
        assert rel_err(dx_a, dx_b) < TOL, (call, rel_err(dx_a, dx_b))
        assert rel_err(dg_a, dg_b) < TOL, (call, rel_err(dg_a, dg_b))


def test_noalloc_rejects_sizes_beyond_its_scratch():
    from midstream_llm_b200 import _lib
    x = torch.zeros(16, 2048, device="cuda", dtype=torch.float16)
    with pytest.raises(_lib.JxError, match="exceeds the built-in scratch limit"):
        _call_noalloc(_lib, x, x, torch.ones(16, device="cuda"), torch.ones(2048, device="cuda"), None,
                      torch.empty_like(x), torch.zeros(2048, device="cuda"), False)
