"""70B-shaped projections in Q4_K on the GPU: d_model 8192, FFN 28672, GQA
with 8 KV heads of 128 (Wq/Wo 8192 x 8192, Wk/Wv 1024 x 8192, gate/up
28672 x 8192, down 8192 x 28672; [n_out x k]), batch 1, at full size against
the oracle, and row-sharded over 2, 4 and 8 ranks (each rank's rows
[floor(r n / N), floor((r + 1) n / N)), as hesa-llm_b200/sharding.py splits
them) with the shards reassembling the unsharded result.

The down projection's rows (k = 28672) are longer than the strip kernel takes,
so it exercises the streaming kernel at full size."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-5

SHAPES = [
    ("wq_wo", 8192, 8192),
    ("wk_wv", 1024, 8192),
    ("gate_up", 28672, 8192),
    ("down", 8192, 28672),
]


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.fixture(scope="module")
def env():
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import hesa_cuda as H
    import sharding as S
    H.lib()
    return torch, H, S


@pytest.mark.parametrize("name,n_out,k", SHAPES, ids=[s[0] for s in SHAPES])
def test_proj70b_full_and_row_sharded(env, name, n_out, k):
    torch, H, S = env
    rng = np.random.default_rng(7000 + n_out + k)
    w = (rng.standard_normal((n_out, k), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    blocks = O.quantize(O.Q4_K, w)
    del w
    x = rng.standard_normal(k, dtype=np.float32)
    ref = O.qmatvec(O.Q4_K, blocks, x)

    wd = torch.from_numpy(blocks).cuda()
    xd = torch.from_numpy(x).cuda()
    y = H.qmatvec(O.Q4_K, wd, xd).cpu().numpy()
    assert rel_l2(y, ref) <= REL_L2_TOL, f"{name}: rel L2 {rel_l2(y, ref):.3e}"

    strip = k <= 24576   # rows the strip kernel takes: a row's sum does not depend on its neighbours
    for world in (2, 4, 8):
        parts = []
        for rank in range(world):
            r0, r1 = S.row_range(n_out, rank, world)
            ys = H.qmatvec(O.Q4_K, wd[r0:r1], xd).cpu().numpy()
            assert rel_l2(ys, ref[r0:r1]) <= REL_L2_TOL, f"{name} world {world} rank {rank}"
            parts.append(ys)
        got = np.concatenate(parts)
        assert got.shape == (n_out,)
        if strip:
            assert np.array_equal(got.view(np.uint32), y.view(np.uint32)), f"{name} world {world}"
        else:
            assert rel_l2(got, ref) <= REL_L2_TOL
    assert H.device_status() == 0
