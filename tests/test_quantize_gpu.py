"""The GPU block quantizer (hesa_cuda_quantize) against the oracle's
quantizer: identical bytes for every type on seeded rows at several scales
and on edge rows (zeros, constants, a single spike, tiny and large values,
one-signed rows). The oracle's Q4_0/Q8_0 are pinned to gguf-py (test_oracle)."""
import numpy as np
import pytest

from oracle import oracle as O

QTYPES = {"Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}


def edge_rows(k):
    rows = [np.zeros(k), np.full(k, 0.25), np.full(k, -3.0), np.linspace(-1, 1, k),
            np.abs(O.gaussian((k,), 1.0, 7)), -np.abs(O.gaussian((k,), 1.0, 8)),
            O.gaussian((k,), 1e-30, 9), O.gaussian((k,), 1e3, 10)]
    spike = np.zeros(k)
    spike[k // 3] = 5.0
    rows.append(spike)
    return np.stack(rows).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(QTYPES))
def test_gpu_quantizer_matches_oracle_bytes(name):
    import torch
    import hesa_cuda as H
    qt = QTYPES[name]
    k = 512
    x = np.concatenate([O.gaussian((64, k), 0.02, 31), O.gaussian((16, k), 1.0, 32), edge_rows(k)])
    want = O.quantize(qt, x)
    got = H.quantize(qt, torch.from_numpy(x).cuda()).cpu().numpy()
    assert got.shape == want.shape
    bad = np.nonzero((got != want).any(axis=1))[0]
    assert bad.size == 0, f"{name}: rows {bad[:8]} differ"


@pytest.mark.gpu
def test_gpu_quantizer_strided_rows_and_model_shape():
    import torch
    import hesa_cuda as H
    k = 4096
    x = O.gaussian((40, 2 * k), 0.02, 41)
    xt = torch.from_numpy(x).cuda()[:, :k]          # row stride 2k
    got = H.quantize(12, xt).cpu().numpy()
    assert np.array_equal(got, O.quantize(12, np.ascontiguousarray(x[:, :k])))
