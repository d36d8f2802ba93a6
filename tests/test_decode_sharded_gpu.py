"""One sequence decoded on several GPUs (hesa_cuda_decode_step_sharded,
sharding.ShardedDecoder): heads, their KV caches and row shares of gate|up
and the LM head per rank, Wo and W_down whole on every rank; the attention
output and gate|up reach every rank as tagged 64-bit words stored by the
kernels that make them, and the next kernel waits per word (bounded).

World 1 (one GPU): the sharded step's logits are bit-identical to the
unsharded decode step's and within rel-L2 1e-5 of the oracle, for
consecutive tokens and at the 7B widths (2 layers, vocab 32000, ctx 2048).
World 2 (two GPUs, skipped with fewer): two processes, each holding half of
every layer, end every step with the oracle's logits, bit-identical to the
unsharded step's (every row is summed in the same order on any number of
ranks)."""
import os
import socket
import tempfile

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

CFG = dict(n_layer=2, d_model=256, n_head=4, n_kv_head=2, head_dim=64, d_ff=512, vocab=384, ctx=64,
           rms_eps=1e-6, rope_base=10000.0, qtype=O.Q4_K)


def rel_l2(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def host_model(cfg, seed=7, prefill=40):
    import test_decode_step_gpu as T
    return T.build_model(cfg["qtype"], seed=seed, prefill=prefill, cfg={k: v for k, v in cfg.items() if k != "qtype"})


def device_full(c, layers, out_norm, w_out, dev):
    """The unsharded model on `dev` in the decode step's joined layout."""
    import torch
    import hesa_cuda as H
    per = []
    for w in layers:
        qkv = torch.from_numpy(np.concatenate([w["wq"], w["wk"], w["wv"]])).to(dev)
        gu = torch.from_numpy(np.concatenate([w["w_gate"], w["w_up"]])).to(dev)
        nq, nk, nf = w["wq"].shape[0], w["wk"].shape[0], w["w_gate"].shape[0]
        d = dict(wq=qkv[:nq], wk=qkv[nq:nq + nk], wv=qkv[nq + nk:], w_gate=gu[:nf], w_up=gu[nf:], _k=(qkv, gu))
        for n in ("wo", "w_down", "attn_norm", "ffn_norm"):
            d[n] = torch.from_numpy(w[n]).to(dev)
        for n in ("k_cache", "v_cache"):
            d[n] = torch.from_numpy(w[n].view(np.int16)).to(dev)
        per.append(d)
    table = torch.from_numpy(H.rope_table(2 * c["ctx"] + 128, c["head_dim"], c["rope_base"])).to(dev)
    return dict(layers=per, w_out=torch.from_numpy(w_out).to(dev), out_norm=torch.from_numpy(out_norm).to(dev),
                table=table)


def test_world1_matches_unsharded_step_and_oracle():
    import torch
    import hesa_cuda as H
    import sharding
    c, layers, out_norm, w_out, emb = host_model(CFG)
    full = device_full(c, layers, out_norm, w_out, "cuda")
    dec = sharding.ShardedDecoder(c, full, 0, 1, device="cuda")
    # the unsharded step on its own copy of the caches
    ref = device_full(c, layers, out_norm, w_out, "cuda")
    m = H.Model(c["n_layer"], c["d_model"], c["n_head"], c["n_kv_head"], c["head_dim"], c["d_ff"], c["vocab"],
                c["ctx"], c["rms_eps"], c["rope_base"], c["qtype"])
    ws = H.decode_workspace(m)
    lg = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    emb_d = torch.from_numpy(emb).cuda()
    for pos, tok in [(40, 5), (41, 77), (42, 383), (80, 9)]:   # the last one wraps the 64-slot ring
        pos_dev = torch.tensor([pos], dtype=torch.int32, device="cuda")
        tok_dev = torch.tensor([tok], dtype=torch.int32, device="cuda")
        x = H.embed(c["qtype"], emb_d, c["d_model"], tok_dev)
        dec.step(x, pos_dev)
        H.decode_step(m, H.make_layers(ref["layers"]), ref["out_norm"], ref["w_out"], ref["table"], x, pos_dev,
                      lg, ws)
        torch.cuda.synchronize()
        got = dec.logits().cpu().numpy()
        assert np.array_equal(got.view(np.uint32), lg.cpu().numpy().view(np.uint32)), pos
        x_ref = O.dequantize(c["qtype"], emb[tok:tok + 1], c["d_model"])[0]
        want = O.decode_step(c, layers, out_norm, w_out, x_ref, pos)
        assert rel_l2(got, want) <= 1e-5, pos
    assert H.device_status() == 0
    dec.close()


def test_world1_7b_widths_match_unsharded_step():
    import torch
    import hesa_cuda as H
    import sharding
    import test_decode_7b_gpu as T7
    cfg = dict(T7.CFG_7B, n_layer=2)
    dev_layers, _, w_out, emb, out_norm = T7.build(cfg, seed=31)
    table = torch.from_numpy(H.rope_table(cfg["ctx"], cfg["head_dim"], cfg["rope_base"])).cuda()
    full = dict(layers=dev_layers, w_out=w_out, out_norm=out_norm, table=table)
    dec = sharding.ShardedDecoder(cfg, full, 0, 1, device="cuda")   # copies the caches it shards
    m = H.Model(cfg["n_layer"], cfg["d_model"], cfg["n_head"], cfg["n_kv_head"], cfg["head_dim"], cfg["d_ff"],
                cfg["vocab"], cfg["ctx"], cfg["rms_eps"], cfg["rope_base"], cfg["qtype"])
    ws = H.decode_workspace(m)
    lg = torch.empty(cfg["vocab"], dtype=torch.float32, device="cuda")
    pos_dev = torch.tensor([T7.POS], dtype=torch.int32, device="cuda")
    x = H.embed(cfg["qtype"], emb, cfg["d_model"], torch.tensor([1234], dtype=torch.int32, device="cuda"))
    dec.step(x, pos_dev)
    H.decode_step(m, H.make_layers(dev_layers), out_norm, w_out, table, x, pos_dev, lg, ws)
    torch.cuda.synchronize()
    assert torch.equal(dec.logits(), lg)
    assert H.device_status() == 0
    dec.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg_for(world):
    """The small model, with as many heads as the ranks need (8 of 64 for
    more than two ranks)."""
    return CFG if world <= 2 else dict(CFG, d_model=512, n_head=8, n_kv_head=8, d_ff=1024)


def _rank_main(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "hesa-llm_b200"), os.path.join(root, "tests")]
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    import hesa_cuda as H
    import sharding
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        c, layers, out_norm, w_out, emb = host_model(_cfg_for(world))
        full = device_full(c, layers, out_norm, w_out, dev)
        dec = sharding.ShardedDecoder(c, full, rank, world, device=dev)
        emb_d = torch.from_numpy(emb).to(dev)
        torch.cuda.synchronize(dev)
        dist.barrier()   # the ranks start their first step within the peer wait limit of one another
        for pos, tok in [(40, 5), (41, 77), (42, 383)]:
            pos_dev = torch.tensor([pos], dtype=torch.int32, device=dev)
            tok_dev = torch.tensor([tok], dtype=torch.int32, device=dev)
            x = H.embed(c["qtype"], emb_d, c["d_model"], tok_dev)
            dec.step(x, pos_dev)
            torch.cuda.synchronize(dev)
            np.save(os.path.join(out_dir, f"r{rank}_p{pos}.npy"), dec.logits().cpu().numpy())
        np.save(os.path.join(out_dir, f"status{rank}.npy"), np.array([H.device_status()]))
        dist.barrier()
        dec.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gpus_decode_one_sequence(world):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, world, port, d)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        import hesa_cuda as H
        c, layers, out_norm, w_out, emb = host_model(_cfg_for(world))
        ref = device_full(c, layers, out_norm, w_out, "cuda:0")
        m = H.Model(c["n_layer"], c["d_model"], c["n_head"], c["n_kv_head"], c["head_dim"], c["d_ff"], c["vocab"],
                    c["ctx"], c["rms_eps"], c["rope_base"], c["qtype"])
        ws = H.decode_workspace(m)
        lg = torch.empty(c["vocab"], dtype=torch.float32, device="cuda:0")
        emb_d = torch.from_numpy(emb).to("cuda:0")
        for pos, tok in [(40, 5), (41, 77), (42, 383)]:
            x_ref = O.dequantize(c["qtype"], emb[tok:tok + 1], c["d_model"])[0]
            want = O.decode_step(c, layers, out_norm, w_out, x_ref, pos)
            r0 = np.load(os.path.join(d, f"r0_p{pos}.npy"))
            for r in range(1, world):
                assert np.array_equal(r0, np.load(os.path.join(d, f"r{r}_p{pos}.npy"))), (pos, r)
            assert rel_l2(r0, want) <= 1e-5, pos
            # the unsharded step on one GPU, same token sequence
            x = H.embed(c["qtype"], emb_d, c["d_model"], torch.tensor([tok], dtype=torch.int32, device="cuda:0"))
            H.decode_step(m, H.make_layers(ref["layers"]), ref["out_norm"], ref["w_out"], ref["table"], x,
                          torch.tensor([pos], dtype=torch.int32, device="cuda:0"), lg, ws)
            torch.cuda.synchronize()
            assert np.array_equal(r0.view(np.uint32), lg.cpu().numpy().view(np.uint32)), pos
        for r in range(world):
            assert int(np.load(os.path.join(d, f"status{r}.npy"))[0]) == 0, r
