"""Row-sharded matvec with the all-gather fused into the kernel
(hesa_cuda_qmatvec_gather + hesa_cuda_peer_barrier, hesa-llm_b200/sharding.py)
on the GPU.

One GPU (world 1): the gathered rows equal the plain matvec bit for bit and
the oracle within rel-L2 1e-5; consecutive steps alternate the two output
parities; several matvecs share one buffer at row offsets; the step replays
from a CUDA graph with the parity following the device-side barrier count.
Two GPUs (skipped with fewer): two processes, each holding half of W's rows,
both end every step with the full y of the oracle. A barrier whose peer never
arrives gives up after the configured wait and reports device status 4.

The tagged form (hesa_cuda_qmatvec_gather_tagged + hesa_cuda_peer_collect,
sharding.TaggedGather): the collected rows equal the plain matvec bit for bit
on one GPU, eagerly and from graph replays, with the step count advancing
once per collect; a collect whose words never arrive reports status 4 after
the configured wait; 2, 4 or 8 processes (skipped without the GPUs) each end
every step with the oracle's full y."""
import os
import socket
import tempfile

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


def test_world1_matches_plain_matvec_and_oracle(torch_cuda):
    torch = torch_cuda
    import hesa_cuda as H
    import sharding as S
    qt, n, k = O.Q4_K, 1000, 4096
    blocks = O.quantize(qt, O.gaussian((n, k), 0.02, 11))
    w = torch.from_numpy(blocks).cuda()
    mv = S.GatheredQMatvec(qt, w, n, k, 0, 1)
    ys = []
    for step in range(3):
        x = O.gaussian((k,), 1.0, 20 + step)
        xt = torch.from_numpy(x).cuda()
        y = mv(xt, scale=0.5).clone()
        torch.cuda.synchronize()
        plain = H.qmatvec(qt, w, xt, scale=0.5)
        assert torch.equal(y, plain)
        assert rel_l2(y.cpu().numpy(), O.qmatvec(qt, blocks, x, scale=0.5)) <= REL_L2_TOL
        ys.append(y)
    # three barriers: the device count is 3, step 2 sits in parity 0, step 1 in parity 1
    epoch = H.device_view(mv.peers.epoch, 1, dtype="<i4")
    assert int(epoch[0]) == 3
    assert torch.equal(mv.peers.output(0)[:n], ys[2]) and torch.equal(mv.peers.output(1)[:n], ys[1])
    assert H.device_status() == 0
    mv.peers.close()


def test_world1_shared_buffer_and_graph_replay(torch_cuda):
    torch = torch_cuda
    import hesa_cuda as H
    import sharding as S
    mats = [(O.Q8_0, 300, 512), (O.Q6_K, 256, 1024), (O.Q5_K, 516, 2048)]
    total = sum(n for _, n, _ in mats)
    peers = S.PeerGather(total, 0, 1)
    mvs, blocks, xs = [], [], []
    off = 0
    for i, (qt, n, k) in enumerate(mats):
        b = O.quantize(qt, O.gaussian((n, k), 0.02, 40 + i))
        blocks.append(b)
        xs.append(torch.from_numpy(O.gaussian((k,), 1.0, 50 + i)).cuda())
        mvs.append(S.GatheredQMatvec(qt, torch.from_numpy(b).cuda(), n, k, 0, 1, peers=peers, row_offset=off))
        off += n
    stream = torch.cuda.Stream()

    def step():
        for mv, x in zip(mvs, xs):
            mv.launch(x, stream=stream)
        H.peer_barrier(peers.flags, 0, 1, peers.epoch, stream=stream)

    with torch.cuda.stream(stream):
        step()                                  # parity 0
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()                              # captured: runs at whatever the count is
    stream.synchronize()
    # capture does not run the kernels: one barrier so far
    for _ in range(4):
        graph.replay()                          # counts 1..4 -> parities 1, 0, 1, 0
    stream.synchronize()
    assert int(H.device_view(peers.epoch, 1, dtype="<i4")[0]) == 5
    for par in (0, 1):
        got = peers.output(par).cpu().numpy()
        off = 0
        for (qt, n, k), b, x in zip(mats, blocks, xs):
            assert rel_l2(got[off:off + n], O.qmatvec(qt, b, x.cpu().numpy())) <= REL_L2_TOL
            off += n
    del graph
    assert H.device_status() == 0
    peers.close()


def test_barrier_wait_runs_out_and_reports_status_4(torch_cuda):
    """A barrier whose peer never arrives (world 2, the peer's flag array a
    local buffer nobody writes) gives up after the wait limit, records device
    status 4 and returns; the context stays usable and the next barrier works."""
    import time
    import hesa_cuda as H
    torch = torch_cuda
    own = torch.zeros(2, dtype=torch.int32, device="cuda")
    fake_peer = torch.zeros(2, dtype=torch.int32, device="cuda")
    epoch = torch.zeros(1, dtype=torch.int32, device="cuda")
    H.clear_device_status()
    H.set_peer_wait_limit(0.05)
    try:
        t0 = time.time()
        H.peer_barrier([own.data_ptr(), fake_peer.data_ptr()], 0, 2, epoch.data_ptr())
        status = H.device_status()
        elapsed = time.time() - t0
        assert status == 4, status
        assert elapsed < 1.5, f"the wait took {elapsed:.2f} s, not the 0.05 s limit"
        # this rank published its arrival into its slot of the peer's array and
        # counted the step as ended
        assert fake_peer.cpu().tolist() == [1, 0]
        assert int(epoch.item()) == 1
    finally:
        H.set_peer_wait_limit(0)
        H.clear_device_status()
    assert H.device_status() == 0
    H.peer_barrier([own.data_ptr()], 0, 1, epoch.data_ptr())     # world 1: completes at once
    assert H.device_status() == 0 and int(epoch.item()) == 2


def test_peer_wait_limit_rejects_values_above_a_minute(torch_cuda):
    import hesa_cuda as H
    with pytest.raises(H.HesaError) as ei:
        H.set_peer_wait_limit(61.0)
    assert ei.value.code == 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_tagged_world1_matches_plain_matvec_and_replays(torch_cuda):
    torch = torch_cuda
    import hesa_cuda as H
    import sharding as S
    # the last shape has longer rows than the strip kernel takes: plain
    # matvec into the workspace, then the scatter kernel
    mats = [(O.Q8_0, 300, 512), (O.Q6_K, 256, 1024), (O.Q4_K, 1000, 4096), (O.Q4_0, 77, 256), (O.Q4_K, 40, 28672)]
    total = sum(n for _, n, _ in mats)
    tg = S.TaggedGather(total, 0, 1, device="cuda")
    assert H.gather_tagged_workspace(O.Q4_K, 1000, 4096) is None
    gws = H.gather_tagged_workspace(O.Q4_K, 40, 28672)
    assert gws is not None
    ws, blocks, xs, tg_targets = [], [], [], []
    off = 0
    for i, (qt, n, k) in enumerate(mats):
        b = O.quantize(qt, O.gaussian((n, k), 0.02, 140 + i))
        blocks.append(b)
        ws.append(torch.from_numpy(b).cuda())
        xs.append(torch.from_numpy(O.gaussian((k,), 1.0, 150 + i)).cuda())
        tg_targets.append(off)
        off += n
    stream = torch.cuda.Stream()

    def step():
        for (qt, n, k), w, x, row0 in zip(mats, ws, xs, tg_targets):
            H.qmatvec_gather_tagged(qt, w, x, tg.targets(), row0, 1, tg.sync, scale=0.25,
                                    workspace=gws if k > 24576 else None, stream=stream)
        tg.collect(stream=stream)

    want = np.concatenate([O.qmatvec(qt, b, x.cpu().numpy(), scale=0.25) for (qt, n, k), b, x in
                           zip(mats, blocks, xs)])
    plain = torch.cat([H.qmatvec(qt, w, x, scale=0.25) for (qt, n, k), w, x in zip(mats, ws, xs)])
    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
        stream.synchronize()
        assert torch.equal(tg.out, plain)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        tg.out.zero_()
        for _ in range(5):
            graph.replay()
    stream.synchronize()
    assert int(H.device_view(tg.sync, 1, dtype="<i4")[0]) == 8   # 3 eager + 5 replays
    assert int(H.device_view(tg.sync + 4, 1, dtype="<i4")[0]) == 0
    assert torch.equal(tg.out, plain)
    assert rel_l2(tg.out.cpu().numpy(), want) <= REL_L2_TOL
    del graph
    assert H.device_status() == 0
    tg.close()


def test_tagged_collect_wait_runs_out_and_reports_status_4(torch_cuda):
    torch = torch_cuda
    import time
    import hesa_cuda as H
    import sharding as S
    tg = S.TaggedGather(1000, 0, 1, device="cuda")
    H.set_peer_wait_limit(0.05)
    try:
        t0 = time.time()
        tg.collect()            # nothing stored this step's words: every wait runs out once
        st = H.device_status()
        assert st == 4, st
        assert time.time() - t0 < 10
    finally:
        H.set_peer_wait_limit(0)
        H.clear_device_status()
    # the context stays usable: a real step afterwards (count 1, parity 1)
    qt, n, k = O.Q4_K, 1000, 1024
    b = O.quantize(qt, O.gaussian((n, k), 0.02, 160))
    x = O.gaussian((k,), 1.0, 161)
    w = torch.from_numpy(b).cuda()
    H.qmatvec_gather_tagged(qt, w, torch.from_numpy(x).cuda(), tg.targets(), 0, 1, tg.sync)
    y = tg.collect()
    torch.cuda.synchronize()
    assert rel_l2(y.cpu().numpy(), O.qmatvec(qt, b, x)) <= REL_L2_TOL
    assert H.device_status() == 0
    tg.close()


def _rank_main(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "hesa-llm_b200")]
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    status = "fail"
    try:
        from oracle import oracle as Orc
        import hesa_cuda as H
        import sharding as S
        qt, n, k = Orc.Q4_K, 4100, 4096
        blocks = Orc.quantize(qt, Orc.gaussian((n, k), 0.02, 61))
        r0, r1 = S.row_range(n, rank, world)
        mv = S.GatheredQMatvec(qt, torch.from_numpy(blocks[r0:r1]).cuda(), n, k, rank, world)
        errs = []
        for step in range(3):
            x = Orc.gaussian((k,), 1.0, 70 + step)
            dist.barrier()
            y = mv(torch.from_numpy(x).cuda()).cpu().numpy()
            errs.append(rel_l2(y, Orc.qmatvec(qt, blocks, x)))
        ok = max(errs) <= REL_L2_TOL and H.device_status() == 0
        dist.barrier()
        mv.peers.close()
        status = "ok" if ok else f"errors {errs}"
    finally:
        with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
            f.write(status)
        dist.destroy_process_group()


def _tagged_rank_main(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "hesa-llm_b200")]
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    status = "fail"
    try:
        from oracle import oracle as Orc
        import hesa_cuda as H
        import sharding as S
        mats = [(Orc.Q4_K, 4100, 4096), (Orc.Q6_K, 515, 1024)]
        total = sum(n for _, n, _ in mats)
        tg = S.TaggedGather(total, rank, world, device="cuda")
        shards = []
        off = 0
        for i, (qt, n, k) in enumerate(mats):
            blocks = Orc.quantize(qt, Orc.gaussian((n, k), 0.02, 170 + i))
            r0, r1 = S.row_range(n, rank, world)
            shards.append((qt, n, k, blocks, torch.from_numpy(blocks[r0:r1]).cuda(), off + r0))
            off += n
        dist.barrier()
        errs = []
        for step in range(4):    # both parities twice, ranks not in lockstep between steps
            xs = [Orc.gaussian((k,), 1.0, 180 + 10 * step + i) for i, (_, _, k) in enumerate(mats)]
            for (qt, n, k, blocks, w, row0), x in zip(shards, xs):
                H.qmatvec_gather_tagged(qt, w, torch.from_numpy(x).cuda(), tg.targets(), row0, world, tg.sync)
            y = tg.collect().cpu().numpy()
            want = np.concatenate([Orc.qmatvec(qt, blocks, x) for (qt, n, k, blocks, w, t), x in zip(shards, xs)])
            errs.append(rel_l2(y, want))
        ok = max(errs) <= REL_L2_TOL and H.device_status() == 0
        torch.cuda.synchronize()
        dist.barrier()
        tg.close()
        status = "ok" if ok else f"errors {errs}"
    finally:
        with open(os.path.join(out_dir, f"r{rank}.txt"), "w") as f:
            f.write(status)
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_gpus_tagged_gather_the_full_output(torch_cuda, world):
    torch = torch_cuda
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_tagged_rank_main, args=(r, world, port, d)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            if p.is_alive():
                p.kill()
                pytest.fail("rank did not finish")
        for r in range(world):
            assert open(os.path.join(d, f"r{r}.txt")).read() == "ok", r


def test_two_gpus_gather_the_full_output(torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, 2, port, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(180)
            if p.is_alive():
                p.kill()
                pytest.fail("rank did not finish")
        for r in range(2):
            assert open(os.path.join(d, f"r{r}.txt")).read() == "ok", r
