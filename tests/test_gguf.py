"""GGUF files straight to the GPU (hesa-llm_b200/backend/gguf_file.cpp,
device_model.cpp): the repair of the reference's GGUF parser
(src/model/gguf_loader.cpp:138-272) and device-resident weights.

CPU: files written by the gguf Python package (GGUFWriter; third party,
independent of this code) with every metadata value type -- arrays of
strings, integers and floats, 8- and 16-bit integers, booleans, a float RMS
epsilon, 64-bit values, a custom alignment -- and quantized and F32 tensors
parse to exactly what was written (values, tensor shapes, types, data
offsets, checked against the package's own reader too). Truncated and corrupt
files are refused with INVALID_FORMAT (8), never read out of bounds. The
reference's parser desynchronises on such files: it skips 4 bytes for the
value types it does not decode (gguf_loader.cpp:184-187) and aligns before the
tensor infos (:249).

GPU: a small Llama-shaped Q4_K model written as GGUF is uploaded once
(DeviceModel), every projection runs through hesa::CudaBackend::matmul as a
device-resident view (batch 1 and 3) within rel-L2 1e-5 of the oracle, and a
DecodeSession decodes tokens from position 0 with logits within rel-L2 1e-5
of the oracle's decode step."""
import json
import os
import subprocess
import tempfile

import numpy as np
import pytest

from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "hesa-llm_b200")
OUT_DIR = os.path.join(ROOT, "tests", "cpp", "_build")
DUMP = os.path.join(OUT_DIR, "gguf_dump")
GPU_EXE = os.path.join(OUT_DIR, "test_gguf_gpu")
REF_SRC = os.path.join(ROOT, "oracle", "_ref", "src")


def _stale(target, inputs):
    return not os.path.exists(target) or any(os.path.getmtime(p) > os.path.getmtime(target) for p in inputs)


def build_dump() -> str:
    srcs = [os.path.join(ROOT, "tests", "cpp", "gguf_dump.cpp"), os.path.join(PKG, "backend", "gguf_file.cpp")]
    if _stale(DUMP, srcs + [os.path.join(PKG, "backend", "gguf_file.hpp")]):
        os.makedirs(OUT_DIR, exist_ok=True)
        res = subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", "-I", PKG, *srcs, "-o", DUMP],
                             capture_output=True, text=True)
        assert res.returncode == 0, res.stderr[-4000:]
    return DUMP


def build_gpu_program() -> str:
    if not os.path.isdir(REF_SRC):
        pytest.skip("the reference's Tensor sources are not prepared (oracle/_ref/src)")
    import hesa_cuda as H
    H.lib()
    cuda_lib = H.library_path()
    srcs = [os.path.join(ROOT, "tests", "cpp", "test_gguf_gpu.cpp")] + [
        os.path.join(PKG, "backend", f) for f in ("gguf_file.cpp", "device_model.cpp", "cuda_backend.cpp")] + [
        os.path.join(REF_SRC, "src", "tensor", "tensor.cpp")]
    hdrs = [os.path.join(PKG, "backend", f) for f in ("gguf_file.hpp", "device_model.hpp", "cuda_backend.hpp")]
    if _stale(GPU_EXE, srcs + hdrs + [cuda_lib, os.path.join(ROOT, "include", "hesa_cuda.h")]):
        os.makedirs(OUT_DIR, exist_ok=True)
        cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
        cmd = ["g++", "-std=c++23", "-O2", "-pthread", "-include", "algorithm", "-include", "cstring",
               "-DHESA_ARCH_x86_64=1", "-DHESA_PLATFORM_linux=1",
               "-I", os.path.join(REF_SRC, "include"), "-I", os.path.join(REF_SRC, "src"), "-I", PKG,
               "-I", os.path.join(ROOT, "include"), "-I", os.path.join(cuda_home, "include"), *srcs, "-o", GPU_EXE,
               "-L", os.path.dirname(cuda_lib), "-lhesa_cuda", "-L", os.path.join(cuda_home, "lib64"), "-lcudart",
               "-Wl,-rpath," + os.path.dirname(cuda_lib)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        assert res.returncode == 0, res.stderr[-4000:]
    return GPU_EXE


def dump(path):
    res = subprocess.run([build_dump(), path], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    return json.loads(res.stdout)


def write_gguf(path, tensors, kv=None, alignment=None, arch="llama"):
    """tensors: list of (name, array, raw qtype or None)."""
    import gguf
    w = gguf.GGUFWriter(path, arch)
    if alignment:
        w.add_custom_alignment(alignment)
    for fn, args in (kv or []):
        getattr(w, fn)(*args)
    for name, arr, qt in tensors:
        if qt is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=gguf.GGMLQuantizationType(qt))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


ALL_KV = [
    ("add_uint8", ("t.u8", 200)), ("add_int8", ("t.i8", -100)), ("add_uint16", ("t.u16", 60000)),
    ("add_int16", ("t.i16", -30000)), ("add_uint32", ("t.u32", 4000000000)), ("add_int32", ("t.i32", -2000000000)),
    ("add_float32", ("t.f32", 0.15625)), ("add_bool", ("t.bool", True)), ("add_string", ("t.str", "héllo \"x\"")),
    ("add_uint64", ("t.u64", 2 ** 63 + 5)), ("add_int64", ("t.i64", -(2 ** 40))), ("add_float64", ("t.f64", 1e-300)),
    ("add_array", ("t.arr_str", ["a", "", "bc", "déf"])), ("add_array", ("t.arr_int", [1, -2, 3])),
    ("add_array", ("t.arr_f", [0.5, -1.25])),
    ("add_block_count", (2,)), ("add_embedding_length", (512,)), ("add_feed_forward_length", (1024,)),
    ("add_head_count", (8,)), ("add_head_count_kv", (2,)), ("add_layer_norm_rms_eps", (1e-6,)),
    ("add_rope_freq_base", (500000.0,)), ("add_context_length", (4096,)),
    ("add_array", ("tokenizer.ggml.tokens", [f"tok{i}" for i in range(300)])),
]


def sample_tensors():
    qk = O.quantize(O.Q4_K, O.gaussian((37, 512), 0.02, 1))
    q8 = O.quantize(O.Q8_0, O.gaussian((64, 96), 0.02, 2))
    q6 = O.quantize(O.Q6_K, O.gaussian((3, 2, 256), 0.02, 3).reshape(6, 256)).reshape(3, 2, 210)
    f32 = O.gaussian((512,), 1.0, 4)
    f16 = O.gaussian((5, 7), 1.0, 5).astype(np.float16)
    return [("blk.0.attn_q.weight", qk, O.Q4_K), ("q8", q8, O.Q8_0), ("q6_3d", q6, O.Q6_K),
            ("blk.0.attn_norm.weight", f32, None), ("h16", f16, None)]


@pytest.mark.parametrize("alignment", [None, 64])
def test_parses_every_value_type_and_tensor(alignment):
    import gguf
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        tensors = sample_tensors()
        write_gguf(path, tensors, ALL_KV, alignment)
        got = dump(path)
        assert got["rc"] == 0, got["error"]
        assert got["version"] == 3 and got["alignment"] == (alignment or 32)
        kv = got["kv"]
        assert kv["t.u8"]["i"] == 200 and kv["t.u8"]["type"] == 0
        assert kv["t.i8"]["i"] == -100 and kv["t.u16"]["i"] == 60000 and kv["t.i16"]["i"] == -30000
        assert kv["t.u32"]["i"] == 4000000000 and kv["t.i32"]["i"] == -2000000000
        assert kv["t.f32"]["f"] == 0.15625 and kv["t.bool"]["i"] == 1
        assert kv["t.str"]["s"] == "héllo \"x\""
        assert kv["t.u64"]["u"] == 2 ** 63 + 5 and kv["t.i64"]["i"] == -(2 ** 40) and kv["t.f64"]["f"] == 1e-300
        assert kv["t.arr_str"]["strings"] == ["a", "", "bc", "déf"] and kv["t.arr_str"]["count"] == 4
        assert kv["t.arr_int"]["ints"] == [1, -2, 3] and kv["t.arr_f"]["floats"] == [0.5, -1.25]
        assert kv["tokenizer.ggml.tokens"]["count"] == 300
        # the float epsilon (the reference reads it as an integer)
        ll = got["llama"]
        assert abs(ll["rms_eps"] - 1e-6) < 1e-12 and ll["rope_base"] == 500000.0
        assert (ll["n_layer"], ll["d_model"], ll["n_head"], ll["n_kv_head"], ll["d_ff"], ll["context"]) == \
            (2, 512, 8, 2, 1024, 4096)
        # tensors against the independent reader of the gguf package
        ref = gguf.GGUFReader(path)
        by_name = {t["name"]: t for t in got["tensors"]}
        assert len(by_name) == len(tensors)
        for rt in ref.tensors:
            t = by_name[rt.name]
            assert t["type"] == int(rt.tensor_type), rt.name
            assert t["ne"][:t["n_dims"]] == [int(v) for v in rt.shape], rt.name
            assert t["file_offset"] == int(rt.data_offset), rt.name
            assert t["bytes"] == int(rt.n_bytes), rt.name
            assert t["file_offset"] % (alignment or 32) == 0
        raw = open(path, "rb").read()
        for name, arr, _ in tensors:
            t = by_name[name]
            assert raw[t["file_offset"]:t["file_offset"] + t["bytes"]] == np.ascontiguousarray(arr).tobytes(), name


def test_refuses_truncated_and_corrupt_files():
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.gguf")
        write_gguf(path, sample_tensors(), ALL_KV)
        raw = open(path, "rb").read()
        good = dump(path)
        data_start = good["data_offset"]
        data_end = max(t["file_offset"] + t["bytes"] for t in good["tensors"])   # the writer pads after it
        cuts = sorted({8, 20, 24, 40, 200, 1000, data_start - 8, data_start + 10, data_end - 1})
        for cut in cuts:
            p = os.path.join(d, f"cut{cut}.gguf")
            open(p, "wb").write(raw[:cut])
            got = dump(p)
            assert got["rc"] == 8, (cut, got)
        bad = bytearray(raw)
        bad[0:4] = b"GGUX"
        open(os.path.join(d, "magic.gguf"), "wb").write(bad)
        assert dump(os.path.join(d, "magic.gguf"))["rc"] == 8
        bad = bytearray(raw)
        bad[4:8] = (1).to_bytes(4, "little")
        open(os.path.join(d, "v1.gguf"), "wb").write(bad)
        assert dump(os.path.join(d, "v1.gguf"))["rc"] == 8
        # an array count far beyond the file: refused before any allocation
        i = raw.index(b"t.arr_int") + len(b"t.arr_int") + 4 + 4
        bad = bytearray(raw)
        bad[i:i + 8] = (2 ** 40).to_bytes(8, "little")
        open(os.path.join(d, "count.gguf"), "wb").write(bad)
        assert dump(os.path.join(d, "count.gguf"))["rc"] == 8
        assert dump(os.path.join(d, "missing.gguf"))["rc"] == 7


# --------------------------------------------------------------------------
# GPU: upload, device-resident matmul, decode from the file
# --------------------------------------------------------------------------

CFG = dict(n_layer=2, d_model=256, n_head=4, n_kv_head=2, head_dim=64, d_ff=512, vocab=384, ctx=64,
           rms_eps=1e-6, rope_base=10000.0, qtype=O.Q4_K)


def llama_file(path, cfg, seed=5):
    """A random Llama-shaped model as GGUF, and the same weights for the oracle."""
    qt = cfg["qtype"]
    D, QD, KD, F, V = cfg["d_model"], cfg["n_head"] * cfg["head_dim"], cfg["n_kv_head"] * cfg["head_dim"], \
        cfg["d_ff"], cfg["vocab"]
    tensors, layers = [], []
    emb = O.quantize(qt, O.gaussian((V, D), 1.0, seed))
    tensors.append(("token_embd.weight", emb, qt))
    for l in range(cfg["n_layer"]):
        s = seed * 100 + 10 * l
        w = {n: O.quantize(qt, O.gaussian(shape, 0.02, s + i)) for i, (n, shape) in enumerate(
            [("wq", (QD, D)), ("wk", (KD, D)), ("wv", (KD, D)), ("wo", (D, QD)), ("w_gate", (F, D)),
             ("w_up", (F, D)), ("w_down", (D, F))])}
        w["attn_norm"] = (1.0 + 0.1 * O.gaussian((D,), 1.0, s + 7)).astype(np.float32)
        w["ffn_norm"] = (1.0 + 0.1 * O.gaussian((D,), 1.0, s + 8)).astype(np.float32)
        w["k_cache"] = np.zeros((cfg["ctx"], KD), np.uint16)
        w["v_cache"] = np.zeros((cfg["ctx"], KD), np.uint16)
        layers.append(w)
        b = f"blk.{l}."
        for gn, key in (("attn_q", "wq"), ("attn_k", "wk"), ("attn_v", "wv"), ("attn_output", "wo"),
                        ("ffn_gate", "w_gate"), ("ffn_up", "w_up"), ("ffn_down", "w_down")):
            tensors.append((b + gn + ".weight", w[key], qt))
        tensors.append((b + "attn_norm.weight", w["attn_norm"], None))
        tensors.append((b + "ffn_norm.weight", w["ffn_norm"], None))
    out_norm = (1.0 + 0.1 * O.gaussian((D,), 1.0, seed + 1)).astype(np.float32)
    w_out = O.quantize(qt, O.gaussian((V, D), 0.02, seed + 2))
    tensors += [("output_norm.weight", out_norm, None), ("output.weight", w_out, qt)]
    kv = [("add_block_count", (cfg["n_layer"],)), ("add_embedding_length", (D,)),
          ("add_feed_forward_length", (F,)), ("add_head_count", (cfg["n_head"],)),
          ("add_head_count_kv", (cfg["n_kv_head"],)), ("add_layer_norm_rms_eps", (cfg["rms_eps"],)),
          ("add_rope_freq_base", (cfg["rope_base"],)), ("add_context_length", (cfg["ctx"],)),
          ("add_array", ("tokenizer.ggml.tokens", [f"t{i}" for i in range(V)]))]
    write_gguf(path, tensors, kv)
    return tensors, layers, out_norm, w_out, emb


def test_gpu_program_builds():
    build_dump()
    assert os.access(build_gpu_program(), os.X_OK)


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


@pytest.mark.gpu
def test_gguf_to_gpu_matmul_and_decode_match_oracle():
    exe = build_gpu_program()
    cfg = CFG
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "llama.gguf")
        tensors, layers, out_norm, w_out, emb = llama_file(path, cfg)
        ks = sorted({arr.shape[1] * O.BLOCK_ELEMS[qt] // O.BLOCK_BYTES[qt] for _, arr, qt in tensors if qt})
        xs = {}
        for k in ks:
            x = O.gaussian((k,), 1.0, 900 + k)
            x3 = O.gaussian((3, k + 4), 1.0, 901 + k)
            x.tofile(os.path.join(d, f"x_{k}.f32"))
            x3.tofile(os.path.join(d, f"x3_{k}.f32"))
            xs[k] = (x, x3)
        steps = [(5, 0), (77, 1), (383, 2), (9, 3)]
        res = subprocess.run([exe, path, d, str(cfg["ctx"])] + [f"{t}@{p}" for t, p in steps],
                             capture_output=True, text=True, timeout=300)
        print(res.stdout)
        assert res.returncode == 0, res.stdout + res.stderr
        n_mm = 0
        for name, arr, qt in tensors:
            if qt is None:
                continue
            k = arr.shape[1] * O.BLOCK_ELEMS[qt] // O.BLOCK_BYTES[qt]
            x, x3 = xs[k]
            y = np.fromfile(os.path.join(d, f"y_{name}.f32"), np.float32)
            assert rel_l2(y, O.qmatvec(qt, arr, x)) <= 1e-5, name
            y3 = np.fromfile(os.path.join(d, f"y3_{name}.f32"), np.float32).reshape(3, -1)[:, :arr.shape[0]]
            want3 = O.qmatvec(qt, arr, x3[:, :k])
            for b in range(3):
                assert rel_l2(y3[b], want3[b]) <= 1e-5, (name, b)
            n_mm += 1
        assert n_mm == 2 + 7 * cfg["n_layer"]
        for tok, pos in steps:
            x_ref = O.dequantize(cfg["qtype"], emb[tok:tok + 1], cfg["d_model"])[0]
            want = O.decode_step(cfg, layers, out_norm, w_out, x_ref, pos)
            got = np.fromfile(os.path.join(d, f"logits_{pos}.f32"), np.float32)
            assert rel_l2(got, want) <= 1e-5, pos
