"""GPU parity of the CUDA matvec and dequantizer against the oracle, through
the C ABI (hesa_cuda -> libhesa_cuda.so).

Bars: dequantized weights bit-exact; matvec
outputs within relative L2 error REL_L2_TOL of the fp32 oracle."""
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-5
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


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


def gpu_qmatvec(torch, qt, blocks, x, scale=1.0, k=None):
    import hesa_cuda as H
    w = torch.from_numpy(np.ascontiguousarray(blocks)).cuda()
    xt = torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()
    y = H.qmatvec(qt, w, xt, scale=scale, k=k)
    torch.cuda.synchronize()
    return y.cpu().numpy()


def seeded(qt, n, k, seed, std=0.02):
    return O.quantize(qt, O.gaussian((n, k), std, seed))


@pytest.mark.parametrize("name", list(O.QTYPES))
def test_golden_dequant_bit_exact(torch_cuda, name):
    import hesa_cuda as H
    g = np.load(os.path.join(GOLDEN, f"dequant_{name}.npz"))
    qt = int(g["qtype"])
    k = O.BLOCK_ELEMS[qt]
    w = torch_cuda.from_numpy(g["blocks"]).cuda()
    out = H.dequantize(qt, w, k).cpu().numpy()
    exp = g["expect"].reshape(out.shape)
    assert np.array_equal(out.view(np.uint32), exp.view(np.uint32))


@pytest.mark.parametrize("name", list(O.QTYPES))
def test_dequant_bit_exact_vs_oracle(torch_cuda, name):
    import hesa_cuda as H
    qt = O.QTYPES[name]
    blocks = seeded(qt, 64, 4096, 11 + qt)
    out = H.dequantize(qt, torch_cuda.from_numpy(blocks).cuda(), 4096).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), O.dequantize(qt, blocks, 4096).view(np.uint32))


@pytest.mark.parametrize("name", list(O.QTYPES))
def test_golden_matvec_reference_matmul(torch_cuda, name):
    """Against y = the reference's own cpu_matmul_f32 on independently decoded
    weights (tests/golden/make_golden.py), batch 3, scale 0.75."""
    g = np.load(os.path.join(GOLDEN, f"matvec_{name}.npz"))
    y = gpu_qmatvec(torch_cuda, int(g["qtype"]), g["blocks"], g["x"], float(g["scale"]))
    assert rel_l2(y, g["y"]) <= REL_L2_TOL


CONFIG_SHAPES = [("Q4_0", 4096, 4096)] + [(t, n, k) for t in ("Q8_0", "Q4_K", "Q5_K", "Q6_K")
                                          for (n, k) in ((4096, 11008), (11008, 4096))]


@pytest.mark.parametrize("name,n_out,k", CONFIG_SHAPES)
def test_config_shapes_match_oracle(torch_cuda, name, n_out, k):
    qt = O.QTYPES[name]
    blocks = seeded(qt, n_out, k, 1000 + qt + n_out)
    x = O.gaussian((k,), 1.0, 2000 + qt + k)
    y = gpu_qmatvec(torch_cuda, qt, blocks, x)
    assert rel_l2(y, O.qmatvec(qt, blocks, x)) <= REL_L2_TOL


EDGE = [
    ("Q4_K", 1, 256),        # tiny: row-wise kernel
    ("Q4_K", 5, 512),        # partial row group
    ("Q4_K", 37, 768),
    ("Q5_K", 4099, 512),
    ("Q6_K", 33, 768),       # 630-byte rows: misaligned row starts
    ("Q6_K", 4097, 1280),
    ("Q4_0", 63, 4160),      # k not a multiple of 256: row-wise kernel
    ("Q8_0", 7, 96),
    ("Q8_0", 129, 2304),
    ("Q4_0", 8, 32768),      # one row group spread over many warps
    ("Q6_K", 8, 32768),
    ("Q4_K", 8, 32768),
]


@pytest.mark.parametrize("name,n_out,k", EDGE)
def test_edge_shapes(torch_cuda, name, n_out, k):
    qt = O.QTYPES[name]
    blocks = seeded(qt, n_out, k, 3000 + n_out + k)
    x = O.gaussian((k,), 1.0, 4000 + k)
    y = gpu_qmatvec(torch_cuda, qt, blocks, x, scale=-1.5)
    assert rel_l2(y, O.qmatvec(qt, blocks, x, scale=-1.5)) <= REL_L2_TOL


@pytest.mark.parametrize("name", list(O.QTYPES))
def test_batched_cuda_core_path(torch_cuda, name):
    qt = O.QTYPES[name]
    blocks = seeded(qt, 300, 1024, 77)
    x = O.gaussian((5, 1024), 1.0, 78)
    y = gpu_qmatvec(torch_cuda, qt, blocks, x)
    assert rel_l2(y, O.qmatvec(qt, blocks, x)) <= REL_L2_TOL


def test_large_activations_and_zero_blocks(torch_cuda):
    qt = O.Q4_K
    blocks = seeded(qt, 256, 2048, 5)
    blocks[7] = 0                       # an all-zero row
    blocks[9, :144] = 0                 # an all-zero super-block
    x = O.gaussian((2048,), 300.0, 6)
    y = gpu_qmatvec(torch_cuda, qt, blocks, x)
    ref = O.qmatvec(qt, blocks, x)
    assert y[7] == 0.0
    assert rel_l2(y, ref) <= REL_L2_TOL


def test_deterministic_and_workspace_left_clean(torch_cuda):
    import hesa_cuda as H
    torch = torch_cuda
    qt, n, k = O.Q5_K, 4096, 11008
    w = torch.from_numpy(seeded(qt, n, k, 9)).cuda()
    x = torch.from_numpy(O.gaussian((k,), 1.0, 10)).cuda()
    ws = H.make_workspace(qt, n, k)
    y1 = H.qmatvec(qt, w, x, workspace=ws).clone()
    y2 = H.qmatvec(qt, w, x, workspace=ws).clone()
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    assert int(ws.count_nonzero()) == 0 or int(ws[: ((n + 3) // 4) * 4].count_nonzero()) == 0
    assert H.device_status() == 0
