"""CPU tests of the C ABI: the library builds and loads, exports every function
include/hesa_cuda.h declares, and rejects bad arguments on the host before
any CUDA call (so these run without a GPU)."""
import ctypes
import os
import re

import pytest

import hesa_cuda as H

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for hdr in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if hdr.endswith(".h"):
            text = open(os.path.join(ROOT, "include", hdr)).read()
            names += re.findall(r"HESA_CUDA_API\s+[\w\s\*]+?\b(hesa_cuda_\w+)\s*\(", text)
    return names


def test_header_declares_the_abi():
    names = declared_functions()
    assert "hesa_cuda_qmatvec" in names and "hesa_cuda_dequantize" in names
    assert sorted(names) == sorted(n for n, _, _ in H.SIGNATURES)


def test_library_exports_every_declared_symbol():
    L = H.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert b"sm_100a" in L.hesa_cuda_version()


@pytest.mark.parametrize("qt,k,expect", [(2, 4096, 2304), (8, 11008, 11696), (12, 11008, 6192),
                                         (13, 4096, 2816), (14, 11008, 9030), (12, 100, 0), (3, 256, 0)])
def test_row_bytes(qt, k, expect):
    assert H.row_bytes(qt, k) == expect


def test_workspace_size_is_small_and_positive():
    ws = H.workspace_bytes(12, 11008, 4096)
    assert 0 < ws < 2 << 20
    assert H.workspace_bytes(3, 16, 256) == 0


def test_batched_workspace_holds_staged_activations():
    # Q4_K / Q5_K at batch >= 2 stage the activations' digit planes in the
    # workspace: 12 KB per unit of 256 (16 rows), 6 KB for up to 8 rows
    one = H.workspace_bytes(12, 4096, 11008, 1)
    b8 = H.workspace_bytes(12, 4096, 11008, 8)
    b16 = H.workspace_bytes(12, 4096, 11008, 16)
    assert one < b8 < b16
    assert b16 >= 43 * 12 * 1024
    assert H.workspace_bytes(12, 4096, 11008, 64) == b16      # 16 rows per launch pair
    # Q8_0 / Q4_0 keep slice partials for their tensor-core path too (8 rows per launch)
    assert H.workspace_bytes(8, 4096, 11008, 16) > H.workspace_bytes(8, 4096, 11008, 1)
    assert H.workspace_bytes(2, 4096, 4096, 3) > H.workspace_bytes(2, 4096, 4096, 1)
    # a type without a batched kernel keeps the batch-1 size
    assert H.workspace_bytes(14, 4096, 11008, 16) == H.workspace_bytes(14, 4096, 11008, 1)


@pytest.mark.parametrize("qt", [2, 8])
def test_block_type_batched_workspace(qt):
    # Q8_0 / Q4_0 take the tensor-core path only for k a multiple of 256: other
    # widths keep the batch-1 size; one plan serves every launch of 8 rows
    one = H.workspace_bytes(qt, 4096, 4096, 1)
    assert H.workspace_bytes(qt, 4096, 4096 + 32, 8) == H.workspace_bytes(qt, 4096, 4096 + 32, 1)
    b3, b8, b64 = (H.workspace_bytes(qt, 4096, 4096, b) for b in (3, 8, 64))
    assert one < b3 == b8 == b64
    # tickets (one int per two rows, 256-byte aligned) plus at least two slices of
    # 8-row partial sums
    assert b8 >= ((4096 + 1) // 2) * 4 + 2 * 4096 * 8 * 4


FAKE = 1 << 20  # non-null, 16-byte aligned, never dereferenced: validation fails first


def call(qt=12, w=FAKE, n=64, k=256, x=FAKE, ldx=256, b=1, y=FAKE, ldy=64, ws=FAKE, wsb=1 << 20):
    return H.lib().hesa_cuda_qmatvec(qt, w, n, k, x, ldx, b, y, ldy, 1.0, ws, wsb, None)


@pytest.mark.parametrize("kwargs,code", [
    (dict(qt=3), 3),                 # unsupported type -> BACKEND_NOT_AVAILABLE
    (dict(w=0), 2),                  # null -> INVALID_ARGUMENT
    (dict(x=0), 2),
    (dict(n=0), 6),                  # SHAPE_MISMATCH
    (dict(k=100), 6),                # not a multiple of the block
    (dict(ldx=128), 6),
    (dict(b=2, ldy=32), 6),
    (dict(w=FAKE + 8), 2),           # misaligned weights
    (dict(x=FAKE + 4), 2),           # misaligned activations
    # k = 32768 takes the split-row kernel, the one that needs the workspace
    (dict(k=32768, ldx=32768, wsb=16), 2),   # workspace too small
    (dict(k=32768, ldx=32768, ws=0), 2),
    # Q4_K at batch >= 2 takes the batched kernel, which needs the workspace
    (dict(b=4, wsb=16), 2),
    (dict(b=4, ws=FAKE + 8), 2),
])
def test_qmatvec_rejects_bad_arguments_without_launching(kwargs, code):
    assert call(**kwargs) == code
    assert H.lib().hesa_cuda_last_error()


def test_dequantize_rejects_bad_arguments():
    L = H.lib()
    assert L.hesa_cuda_dequantize(12, FAKE, 4, 100, FAKE, 100, None) == 6
    assert L.hesa_cuda_dequantize(5, FAKE, 4, 256, FAKE, 256, None) == 3
    assert L.hesa_cuda_dequantize(12, 0, 4, 256, FAKE, 256, None) == 2


def test_quantize_rejects_bad_arguments():
    L = H.lib()
    assert L.hesa_cuda_quantize(5, FAKE, 4, 256, 256, FAKE, None) == 3
    assert L.hesa_cuda_quantize(12, 0, 4, 256, 256, FAKE, None) == 2
    assert L.hesa_cuda_quantize(12, FAKE, 4, 100, 100, FAKE, None) == 6
    assert L.hesa_cuda_quantize(2, FAKE, 4, 64, 32, FAKE, None) == 6


def test_error_type_carries_reference_code():
    with pytest.raises(H.HesaError) as ei:
        H._check(6)
    assert ei.value.code == 6 and "SHAPE_MISMATCH" in str(ei.value)


def gather_call(qt=12, w=FAKE, n=64, k=256, x=FAKE, peers=(FAKE,) * 4, world=2, epoch=FAKE):
    arr = (ctypes.c_void_p * len(peers))(*peers) if peers is not None else None
    return H.lib().hesa_cuda_qmatvec_gather(qt, w, n, k, x, 1.0, arr, world, epoch, None)


@pytest.mark.parametrize("kwargs,code", [
    (dict(qt=3), 3),
    (dict(w=0), 2),
    (dict(x=0), 2),
    (dict(epoch=0), 2),
    (dict(peers=None), 2),
    (dict(world=0), 2),
    (dict(world=9, peers=(FAKE,) * 18), 2),
    (dict(n=0), 6),
    (dict(k=96, qt=2), 6),           # gathered path needs whole 256-weight units
    (dict(w=FAKE + 8), 2),
    (dict(x=FAKE + 4), 2),
])
def test_gathered_matvec_rejects_bad_arguments_without_launching(kwargs, code):
    assert gather_call(**kwargs) == code
    assert H.lib().hesa_cuda_last_error()


def tagged_call(qt=12, w=FAKE, n=64, k=256, x=FAKE, peers=(FAKE,) * 4, row0=0, world=2, sync=FAKE, ws=None,
                ws_bytes=0):
    arr = (ctypes.c_void_p * len(peers))(*peers) if peers is not None else None
    return H.lib().hesa_cuda_qmatvec_gather_tagged(qt, w, n, k, x, 1.0, arr, row0, world, sync, ws, ws_bytes, None)


@pytest.mark.parametrize("kwargs,code", [
    (dict(qt=3), 3),
    (dict(w=0), 2),
    (dict(sync=0), 2),
    (dict(peers=None), 2),
    (dict(world=9, peers=(FAKE,) * 18), 2),
    (dict(n=0), 6),
    (dict(k=96, qt=2), 6),
    (dict(peers=(FAKE, FAKE + 8, FAKE, FAKE)), 2),    # buffers must be 16-byte aligned
    (dict(row0=-1), 2),
    (dict(k=28672), 2),                                # long rows without the workspace they need
    (dict(k=28672, ws=FAKE, ws_bytes=16), 2),          # ... or with too small a one
])
def test_tagged_gather_rejects_bad_arguments_without_launching(kwargs, code):
    assert tagged_call(**kwargs) == code
    assert H.lib().hesa_cuda_last_error()


def test_tagged_gather_workspace_only_for_long_rows():
    L = H.lib()
    assert L.hesa_cuda_gather_tagged_workspace_size(12, 4096, 4096) == 0
    need = L.hesa_cuda_gather_tagged_workspace_size(12, 4096, 28672)
    assert need >= 4 * 4096 and need % 256 == 0
    assert L.hesa_cuda_gather_tagged_workspace_size(3, 4096, 28672) == 0   # unsupported type
    assert L.hesa_cuda_peer_collect(None, 10, 10, FAKE, FAKE, None) == 2
    assert L.hesa_cuda_peer_collect(FAKE, 10, 5, FAKE, FAKE, None) == 6      # parities overlap
    assert L.hesa_cuda_peer_collect(FAKE, 10, 10, FAKE, FAKE, None) == 6     # not whole units of 256
    assert L.hesa_cuda_peer_collect(FAKE, 0, 256, FAKE, FAKE, None) == 6
    assert L.hesa_cuda_peer_collect(FAKE + 8, 10, 256, FAKE, FAKE, None) == 2


def test_peer_barrier_and_alloc_reject_bad_arguments():
    L = H.lib()
    two = (ctypes.c_void_p * 2)(FAKE, FAKE)
    assert L.hesa_cuda_peer_barrier(two, 2, 2, FAKE, None) == 2      # rank outside world
    assert L.hesa_cuda_peer_barrier(two, 0, 0, FAKE, None) == 2
    assert L.hesa_cuda_peer_barrier(two, 0, 9, FAKE, None) == 2
    assert L.hesa_cuda_peer_barrier(two, 0, 2, None, None) == 2
    assert L.hesa_cuda_peer_barrier((ctypes.c_void_p * 2)(FAKE, 0), 0, 2, FAKE, None) == 2
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    assert L.hesa_cuda_peer_alloc(0, ctypes.byref(ptr), handle) == 2
    assert L.hesa_cuda_peer_alloc(256, None, handle) == 2
    assert L.hesa_cuda_peer_open(None, ctypes.byref(ptr)) == 2
    assert L.hesa_cuda_peer_close(None) == 2
    assert L.hesa_cuda_peer_free(None) == 2


def test_peer_wait_limit_setting_is_host_side_and_bounded():
    L = H.lib()
    assert L.hesa_cuda_set_peer_wait_limit_us(61 * 1000 * 1000) == 2   # above a minute
    assert L.hesa_cuda_set_peer_wait_limit_us(50 * 1000) == 0
    assert L.hesa_cuda_set_peer_wait_limit_us(0) == 0                  # back to the 2 s default


def test_nvtx_tracing_switch_leaves_calls_unchanged():
    """HESA_CUDA_NVTX=1 wraps the entry points in NVTX ranges (no tool
    attached here: the ranges are no-ops); argument checks and error codes
    are the same with it on."""
    import subprocess
    import sys
    code = ("import sys; sys.path[:0] = ['hesa-llm_b200']\n"
            "import ctypes, hesa_cuda as H\n"
            "L = H.lib()\n"
            "rc = L.hesa_cuda_qmatvec(3, 1 << 20, 64, 256, 1 << 20, 256, 1, 1 << 20, 64, 1.0, None, 0, None)\n"
            "rc2 = L.hesa_cuda_peer_collect(None, 10, 256, 1 << 20, 1 << 20, None)\n"
            "print(rc, rc2)\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for env in ({"HESA_CUDA_NVTX": "1"}, {"HESA_CUDA_NVTX": "0"}):
        out = subprocess.run([sys.executable, "-c", code], cwd=root, env={**os.environ, **env},
                             capture_output=True, text=True, timeout=300)
        assert out.returncode == 0, out.stderr
        assert out.stdout.split() == ["3", "2"], out.stdout
