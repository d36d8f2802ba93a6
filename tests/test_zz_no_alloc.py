"""GPU test of hesa_cuda_qmatvec_noalloc, the matvec entry point that takes no
workspace and allocates nothing.

It exists for callers that are not allowed to allocate device memory: a
library embedded in a host program that routes every device allocation
through its own pool or budget, or a serving loop that must not allocate
once it is running. Its scratch is a fixed array inside libhesa_cuda.so, so
its results must equal those of hesa_cuda_qmatvec, the entry point whose
scratch comes from the caller, and those of the oracle -- including on a
second call, which finds the array as the first call left it.

This file is collected last on purpose: if it fails, a run that stops at the
first failure has already run every other test.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-5  # the matvec parity bar of the other GPU tests


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def env():
    import torch
    assert torch.cuda.is_available(), "needs a CUDA device"
    import hesa_cuda as H
    return torch, H, H.lib()


@pytest.mark.parametrize("name,n_out,k,batch", [
    # rows longer than 24576 weights: the streaming kernel, scratch in the fixed array
    ("Q4_K", 4096, 28672, 1),   # row groups split across warps
    ("Q6_K", 1000, 32768, 2),
    ("Q8_0", 2051, 25600, 1),
    ("Q5_K", 37, 24832, 1),
    ("Q4_0", 8, 32768, 1),      # one row group spread over many warps
    # shapes the row-strip kernel takes: no scratch, any number of rows
    ("Q4_K", 4096, 11008, 1),
    ("Q4_K", 100000, 512, 1),   # more rows than the fixed array covers for the streaming kernel
])
def test_noalloc_matches_oracle_and_workspace_entry_point_on_two_calls(env, name, n_out, k, batch):
    torch, H, L = env
    qt = O.QTYPES[name]
    blocks = O.quantize(qt, O.gaussian((n_out, k), 0.02, 900 + qt + n_out))
    x = O.gaussian((batch, k), 1.0, 901 + qt + k)
    want = O.qmatvec(qt, blocks, x)
    w = torch.from_numpy(blocks).cuda()
    xt = torch.from_numpy(x).cuda()
    expected = H.qmatvec(qt, w, xt).cpu().numpy()  # caller-provided workspace
    stream = torch.cuda.current_stream().cuda_stream or None
    for call in range(2):
        y = torch.full((batch, n_out), float("nan"), dtype=torch.float32, device="cuda")
        rc = L.hesa_cuda_qmatvec_noalloc(qt, w.data_ptr(), n_out, k, xt.data_ptr(), k, batch,
                                         y.data_ptr(), n_out, 1.0, stream)
        assert rc == 0, L.hesa_cuda_last_error().decode()
        torch.cuda.synchronize()
        got = y.cpu().numpy()
        assert np.isfinite(got).all(), f"call {call}: outputs left unwritten"
        for b in range(batch):
            assert rel_l2(got[b], want[b]) <= REL_L2_TOL, f"call {call}, row {b}: vs the oracle"
        assert rel_l2(got, expected) <= REL_L2_TOL, f"call {call}: vs hesa_cuda_qmatvec"
    assert H.device_status() == 0


def test_noalloc_rejects_more_rows_than_its_scratch_covers(env):
    torch, H, L = env
    # rows of 32768 weights take the streaming kernel, whose scratch is the
    # fixed array: 65537 rows are refused before anything is launched (the
    # buffers are never read)
    w = torch.zeros(16, dtype=torch.uint8, device="cuda")
    x = torch.zeros(32768, dtype=torch.float32, device="cuda")
    y = torch.zeros(16, dtype=torch.float32, device="cuda")
    rc = L.hesa_cuda_qmatvec_noalloc(12, w.data_ptr(), 65537, 32768, x.data_ptr(), 32768, 1,
                                     y.data_ptr(), 65537, 1.0, None)
    assert rc == 6  # SHAPE_MISMATCH
    assert b"65536" in L.hesa_cuda_last_error()
