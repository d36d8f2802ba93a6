"""Batched matvec on the tensor cores (csrc/qmm_tc.cu and, for Q8_0 / Q4_0,
csrc/qmm_tc_blk.cu; tcgen05) through the C ABI: Q4_K, Q5_K, Q8_0 and Q4_0
weights with 2..33 activation rows against the oracle (rel-L2 <= 1e-5
per activation row), at the batched-decode shapes (4096 x 11008 and
11008 x 4096, B in {2, 4, 8, 16}), ragged tiles, one-unit and 128-unit rows,
strided x / y, non-finite activations, determinism, the workspace counters
left at zero, and replay inside a CUDA graph."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-5


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import hesa_cuda
    hesa_cuda.lib()
    return torch


def seeded(qt, n, k, seed, std=0.02):
    return O.quantize(qt, O.gaussian((n, k), std, seed))


def run(torch, qt, blocks, x, scale=1.0, ws=None):
    import hesa_cuda as H
    w = torch.from_numpy(np.ascontiguousarray(blocks)).cuda()
    xt = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    y = H.qmatvec(qt, w, xt, scale=scale, workspace=ws)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def check_rows(y, ref):
    for b in range(ref.shape[0]):
        e = rel_l2(y[b], ref[b])
        assert e <= REL_L2_TOL, f"activation row {b}: rel L2 {e:.3e}"


@pytest.mark.parametrize("name", ["Q4_K", "Q5_K"])
@pytest.mark.parametrize("n_out,k", [(4096, 11008), (11008, 4096)])
@pytest.mark.parametrize("batch", [2, 4, 8, 16])
def test_batched_decode_shapes(torch_cuda, name, n_out, k, batch):
    qt = O.QTYPES[name]
    blocks = seeded(qt, n_out, k, 500 + qt + n_out)
    x = O.gaussian((batch, k), 1.0, 600 + batch + k)
    check_rows(run(torch_cuda, qt, blocks, x), O.qmatvec(qt, blocks, x))


@pytest.mark.parametrize("name,n_out,k,batch", [
    # (n_out a multiple of 4: y rows are n_out floats apart, and the ABI
    # wants that stride 16-byte aligned at batch > 1)
    ("Q4_K", 100, 256, 3),       # one unit per row, ragged row tile
    ("Q4_K", 4100, 512, 9),      # ragged last tile, 9 rows: second n-tile per plane
    ("Q5_K", 36, 768, 16),
    ("Q4_K", 64, 32768, 5),      # 128 K slices of one unit
    ("Q4_K", 64, 32768, 2),      # two rows on the tensor cores (rows too long for the strip kernel)
    ("Q5_K", 132, 28672, 2),
    ("Q4_K", 260, 1024, 18),     # 16 + 2 rows: the second launch has two rows
    ("Q4_K", 300, 1024, 20),     # two launch pairs (16 + 4 rows)
    ("Q5_K", 516, 2048, 33),     # three launch pairs
])
def test_batched_edges(torch_cuda, name, n_out, k, batch):
    qt = O.QTYPES[name]
    blocks = seeded(qt, n_out, k, 700 + n_out)
    x = O.gaussian((batch, k), 1.0, 800 + k)
    check_rows(run(torch_cuda, qt, blocks, x, scale=-0.5), O.qmatvec(qt, blocks, x, scale=-0.5))


@pytest.mark.parametrize("name", ["Q8_0", "Q4_0"])
@pytest.mark.parametrize("n_out,k", [(4096, 11008), (11008, 4096)])
@pytest.mark.parametrize("batch", [3, 8, 16])
def test_block_types_batched_decode_shapes(torch_cuda, name, n_out, k, batch):
    """Q8_0 / Q4_0 on the tensor cores (qmm_tc_blk.cu): one MMA per 32-weight block."""
    qt = O.QTYPES[name]
    blocks = seeded(qt, n_out, k, 510 + qt + n_out)
    x = O.gaussian((batch, k), 1.0, 610 + batch + k)
    check_rows(run(torch_cuda, qt, blocks, x), O.qmatvec(qt, blocks, x))


@pytest.mark.parametrize("name,n_out,k,batch", [
    ("Q8_0", 100, 256, 3),       # one unit per row, ragged row tile
    ("Q4_0", 4100, 768, 9),      # ragged last tile; three units (a one-unit copy); a second launch of one row
    ("Q8_0", 64, 32768, 4),      # many K slices of one unit (rows too long for the strip kernel)
    ("Q4_0", 64, 32768, 2),      # two rows on the tensor cores (the strip kernel does not take k > 24576)
    ("Q8_0", 300, 1024, 20),     # launches of 8 + 8 + 4 rows
])
def test_block_types_batched_edges(torch_cuda, name, n_out, k, batch):
    qt = O.QTYPES[name]
    blocks = seeded(qt, n_out, k, 710 + n_out)
    x = O.gaussian((batch, k), 1.0, 810 + k)
    check_rows(run(torch_cuda, qt, blocks, x, scale=-0.5), O.qmatvec(qt, blocks, x, scale=-0.5))


@pytest.mark.parametrize("name", ["Q8_0", "Q4_0"])
def test_block_types_non_finite_row_determinism_and_counters(torch_cuda, name):
    import hesa_cuda as H
    torch = torch_cuda
    qt, n, k, batch = O.QTYPES[name], 2048, 4096, 6
    blocks = seeded(qt, n, k, 71)
    x = O.gaussian((batch, k), 1.0, 72)
    x[4, 1000] = np.nan
    w = torch.from_numpy(blocks).cuda()
    xt = torch.from_numpy(x).cuda()
    ws = H.make_workspace(qt, n, k, batch)
    y1 = H.qmatvec(qt, w, xt, workspace=ws).clone()
    y2 = H.qmatvec(qt, w, xt, workspace=ws).clone()
    torch.cuda.synchronize()
    assert torch.equal(y1[[0, 1, 2, 3, 5]], y2[[0, 1, 2, 3, 5]])
    assert bool(torch.isnan(y1[4]).all())
    keep = [0, 1, 2, 3, 5]
    check_rows(y1.cpu().numpy()[keep], O.qmatvec(qt, blocks, x[keep]))
    zero_bytes = (((n + 1) // 2) * 4 + 255) // 256 * 256
    assert int(ws[:zero_bytes].count_nonzero()) == 0
    assert H.device_status() == 0


def test_batched_matches_single_rows(torch_cuda):
    """Each activation row of a batch agrees with the batch-1 kernel on it."""
    qt, n, k = O.Q4_K, 2048, 4096
    blocks = seeded(qt, n, k, 31)
    x = O.gaussian((8, k), 1.0, 32)
    yb = run(torch_cuda, qt, blocks, x)
    for b in range(8):
        y1 = run(torch_cuda, qt, blocks, x[b])
        assert rel_l2(yb[b], y1) <= 2e-6


def test_batched_strided_operands(torch_cuda):
    import hesa_cuda as H
    torch = torch_cuda
    qt, n, k, batch = O.Q4_K, 1000, 2048, 6
    blocks = seeded(qt, n, k, 41)
    xs = O.gaussian((batch, k + 64), 1.0, 42)
    w = torch.from_numpy(blocks).cuda()
    xt = torch.from_numpy(xs).cuda()
    y = torch.full((batch, n + 24), 7.0, dtype=torch.float32, device="cuda")
    ws = H.make_workspace(qt, n, k, batch)
    rc = H.lib().hesa_cuda_qmatvec(qt, w.data_ptr(), n, k, xt.data_ptr(), k + 64, batch, y.data_ptr(), n + 24,
                                   ctypes_float(1.25), ws.data_ptr(), ws.numel(), None)
    assert rc == 0
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    check_rows(got[:, :n], O.qmatvec(qt, blocks, xs[:, :k], scale=1.25))
    assert np.all(got[:, n:] == 7.0)      # padding columns untouched


def ctypes_float(v):
    import ctypes
    return ctypes.c_float(v)


def test_batched_non_finite_row_stays_local(torch_cuda):
    qt, n, k = O.Q4_K, 256, 1024
    blocks = seeded(qt, n, k, 51)
    x = O.gaussian((4, k), 1.0, 52)
    x[2, 300] = np.inf
    y = run(torch_cuda, qt, blocks, x)
    assert np.all(np.isnan(y[2]) | np.isinf(y[2]))
    keep = [0, 1, 3]
    check_rows(y[keep], O.qmatvec(qt, blocks, x[keep]))


def test_batched_deterministic_counters_zero_and_graph(torch_cuda):
    import hesa_cuda as H
    torch = torch_cuda
    qt, n, k, batch = O.Q5_K, 4096, 11008, 16
    blocks = seeded(qt, n, k, 61)
    w = torch.from_numpy(blocks).cuda()
    x = torch.from_numpy(O.gaussian((batch, k), 1.0, 62)).cuda()
    ws = H.make_workspace(qt, n, k, batch)
    y1 = H.qmatvec(qt, w, x, workspace=ws).clone()
    y2 = H.qmatvec(qt, w, x, workspace=ws).clone()
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    # the counter region at the start of the workspace is back at zero
    zero_bytes = (((n + 1) // 2) * 4 + 255) // 256 * 256
    assert int(ws[:zero_bytes].count_nonzero()) == 0
    # the same call captured in a graph and replayed on new activations
    y = torch.empty((batch, n), dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        H.qmatvec(qt, w, x, y=y, workspace=ws, stream=stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            H.qmatvec(qt, w, x, y=y, workspace=ws, stream=stream)
    stream.synchronize()
    x2 = O.gaussian((batch, k), 1.0, 63)
    x.copy_(torch.from_numpy(x2))
    graph.replay()
    torch.cuda.synchronize()
    check_rows(y.cpu().numpy(), O.qmatvec(qt, blocks, x2))
    del graph
    assert H.device_status() == 0
