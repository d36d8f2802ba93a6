"""Row sharding over ranks (hesa-llm_b200/sharding.py) on CPU: the row ranges
partition every n_out with shards balanced to one row, and two gloo ranks
that each compute their rows (with the oracle standing in for the CUDA
matvec) all-gather exactly the unsharded result, for uneven and even row
counts."""
import os
import socket
import tempfile

import numpy as np
import pytest

import sharding


@pytest.mark.parametrize("n", [1, 2, 5, 37, 4096, 11008, 32000])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_row_ranges_partition_and_balance(n, world):
    ranges = [sharding.row_range(n, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    sizes = [r1 - r0 for r0, r1 in ranges]
    assert max(sizes) - min(sizes) <= 1
    assert max(sizes) <= sharding.slot_rows(n, world)


def test_row_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        sharding.row_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_out, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "hesa-llm_b200")]
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    import sharding as S
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        k, qt = 512, O.Q4_K
        w = O.quantize(qt, O.gaussian((n_out, k), 0.02, 123))
        x = O.gaussian((k,), 1.0, 124)
        r0, r1 = S.row_range(n_out, rank, world)

        def local(w_rows, xv, y):
            rows = w_rows.numpy()
            if rows.shape[0]:
                y[: rows.shape[0]] = torch.from_numpy(O.qmatvec(qt, rows, xv.numpy()))

        mv = S.ShardedQMatvec(qt, torch.from_numpy(w[r0:r1]), n_out, k, rank, world, device="cpu", local=local)
        y = mv(torch.from_numpy(x))
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_out", [37, 64])
def test_sharded_matvec_two_gloo_ranks(n_out):
    import torch.multiprocessing as mp
    from oracle import oracle as O
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_rank_main, args=(r, 2, port, n_out, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        want = O.qmatvec(O.Q4_K, O.quantize(O.Q4_K, O.gaussian((n_out, 512), 0.02, 123)), O.gaussian((512,), 1.0, 124))
        for r in range(2):
            got = np.load(os.path.join(d, f"y{r}.npy"))
            assert got.shape == (n_out,)
            assert np.array_equal(got, want)


def _leaving_rank_main(rank, world, port, out_dir):
    """Both ranks take one step; then rank 1 leaves (between steps, nothing in
    flight) and rank 0 takes a second step."""
    import sys
    import time
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "hesa-llm_b200")]
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    from oracle import oracle as O
    import sharding as S
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    n_out, k, qt = 37, 256, O.Q4_K
    w = O.quantize(qt, O.gaussian((n_out, k), 0.02, 321))
    x = torch.from_numpy(O.gaussian((k,), 1.0, 322))
    r0, r1 = S.row_range(n_out, rank, world)

    def local(w_rows, xv, y):
        y[: w_rows.shape[0]] = torch.from_numpy(O.qmatvec(qt, w_rows.numpy(), xv.numpy()))

    mv = S.ShardedQMatvec(qt, torch.from_numpy(w[r0:r1]), n_out, k, rank, world, device="cpu", local=local)
    mv(x)                       # step 1, both ranks
    dist.barrier()
    if rank == 1:
        time.sleep(0.5)         # let the last messages of step 1 land, then leave
        os._exit(0)
    time.sleep(1.0)
    t0 = time.time()
    try:
        mv(x)                   # step 2: rank 1 is gone
        outcome = "completed"
    except S.RankFailure:
        outcome = "RankFailure"
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{outcome} {time.time() - t0:.2f}")
    os._exit(0)                 # the group cannot be torn down collectively any more


def test_rank_leaving_between_steps_ends_the_next_step_with_an_error():
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.get_context("spawn")
        port = _free_port()
        procs = [ctx.Process(target=_leaving_rank_main, args=(r, 2, port, d)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(90)
            if p.is_alive():
                p.kill()
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        outcome, seconds = open(os.path.join(d, "rank0.txt")).read().split()
        assert outcome == "RankFailure"
        assert float(seconds) < 30.0
