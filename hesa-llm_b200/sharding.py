"""Row sharding of the quantized matvec over the GPUs of one node.

Output rows of y = W x are independent: rank r holds the contiguous rows
[r0, r1) of W (packed GGUF rows, balanced to one row, the same split the strip
kernel uses between its CTAs), computes y[r0:r1], and the full y is
all-gathered so every rank holds it. Two ways to gather:

* "tagged" (TaggedGather, what the benchmark runs): the matvec kernel itself
  stores its rows into the gathered buffer of every rank over NVLink (CUDA IPC
  mappings) as 64-bit words that carry the step's tag
  (hesa_cuda_qmatvec_gather_tagged), and one collector kernel per step waits
  until its own buffer holds the step's words (hesa_cuda_peer_collect). No
  padding: each rank writes at its own row offset.
* "peer" (PeerGather): the same with fp32 peer stores and one barrier kernel
  per step publishing completion (hesa_cuda_qmatvec_gather,
  hesa_cuda_peer_barrier).
* "nccl": NCCL's all_gather_into_tensor, which wants equal sizes, so every
  rank contributes a slot of ceil(n_out / world) rows and the gathered buffer
  is compacted back to n_out rows with one index_select (a no-op view when
  world divides n_out). Also what the CPU (gloo) tests run.
"""
from __future__ import annotations


class RankFailure(RuntimeError):
    """A peer rank did not take part in a step's collective in time (it left,
    died or hangs): raised instead of waiting for ever."""


def row_range(n_out: int, rank: int, world: int) -> tuple[int, int]:
    """Rows [r0, r1) of rank `rank`: floor(rank * n_out / world) .. for rank + 1."""
    if world < 1 or not 0 <= rank < world or n_out < 0:
        raise ValueError(f"bad shard: n_out={n_out} rank={rank} world={world}")
    return rank * n_out // world, (rank + 1) * n_out // world


def slot_rows(n_out: int, world: int) -> int:
    """Rows of every rank's slot in the gathered buffer."""
    return -(-n_out // world)


class ShardedQMatvec:
    """y = scale * W x with W's rows split over the ranks of `group`.

    w_rows: this rank's packed rows [r1 - r0, row_bytes] (see row_range).
    local: optional f(w_rows, x, y_slot) computing this rank's rows into
    y_slot[: r1 - r0]; the default is this library's CUDA matvec. It exists
    so the sharding and the gather can run on CPU ranks in tests.
    """

    def __init__(self, qtype: int, w_rows, n_out: int, k: int, rank: int, world: int, group=None,
                 device=None, local=None):
        import torch
        self.qtype, self.n_out, self.k, self.rank, self.world, self.group = qtype, n_out, k, rank, world, group
        self.r0, self.r1 = row_range(n_out, rank, world)
        if w_rows.shape[0] != self.r1 - self.r0:
            raise ValueError(f"rank {rank} holds {w_rows.shape[0]} rows, its shard has {self.r1 - self.r0}")
        self.w = w_rows
        self.device = device or w_rows.device
        self.slot = slot_rows(n_out, world)
        self.y_slot = torch.zeros(self.slot, dtype=torch.float32, device=self.device)
        self.y_all = torch.empty(world * self.slot, dtype=torch.float32, device=self.device)
        if world * self.slot == n_out:
            self.index = None
        else:
            idx = [r * self.slot + i for r in range(world) for i in range(row_range(n_out, r, world)[1]
                                                                            - row_range(n_out, r, world)[0])]
            self.index = torch.tensor(idx, dtype=torch.int64, device=self.device)
        self.local = local or self._cuda_local
        self.workspace = None

    def _cuda_local(self, w_rows, x, y):
        import hesa_cuda as H
        n = w_rows.shape[0]
        if n == 0:
            return
        if self.workspace is None:
            self.workspace = H.make_workspace(self.qtype, n, self.k, device=self.device)
        H.qmatvec(self.qtype, w_rows, x, y=y[:n], workspace=self.workspace)

    def __call__(self, x, scale: float = 1.0):
        import torch.distributed as dist
        self.local(self.w, x, self.y_slot)
        if scale != 1.0:
            self.y_slot.mul_(scale)
        try:
            # the process group's timeout bounds the wait for the other ranks
            dist.all_gather_into_tensor(self.y_all, self.y_slot, group=self.group)
        except RuntimeError as e:   # DistBackendError, gloo / NCCL timeouts and closed connections
            raise RankFailure(f"rank {self.rank}: the all-gather of the sharded matvec did not complete "
                              f"(a peer rank left or timed out): {e}") from e
        return self.y_all if self.index is None else self.y_all.index_select(0, self.index)


def _align(n: int, a: int = 256) -> int:
    return (n + a - 1) // a * a


class PeerGather:
    """Gathered output buffers shared by the ranks of one node.

    Each rank allocates (hesa_cuda_peer_alloc) two parities of an `out_rows`
    fp32 buffer, a flag array of `world` slots and its barrier count, and maps
    every other rank's allocation from the CUDA IPC handles exchanged through
    `group`. Matvecs of a step store into parity `step & 1` of every rank
    (PeerGather.targets gives their addresses); barrier() ends the step.
    """

    def __init__(self, out_rows: int, rank: int, world: int, group=None, device=None):
        import torch.distributed as dist
        import hesa_cuda as H
        if not 1 <= world <= 8 or not 0 <= rank < world:
            raise ValueError(f"bad rank {rank} / world {world}")
        self.out_rows, self.rank, self.world = out_rows, rank, world
        self.y_bytes = _align(4 * out_rows)
        self.flag_off = 2 * self.y_bytes
        self.epoch_off = self.flag_off + _align(4 * world)
        self.local, handle = H.peer_alloc(self.epoch_off + 256)
        handles = [handle]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle, group=group)
        self.base = [self.local if p == rank else H.peer_open(handles[p]) for p in range(world)]
        self.flags = [b + self.flag_off for b in self.base]
        self.epoch = self.local + self.epoch_off
        self.steps = 0      # barriers issued from the host (graph replays are counted by the caller)
        self.device = device

    def targets(self, row0: int) -> list[int]:
        """Addresses (parity-major, then rank) where row `row0` of the
        gathered output lives in every rank's buffers."""
        return [b + par * self.y_bytes + 4 * row0 for par in (0, 1) for b in self.base]

    def barrier(self, stream=None) -> None:
        import hesa_cuda as H
        H.peer_barrier(self.flags, self.rank, self.world, self.epoch, stream=stream)
        self.steps += 1

    def output(self, parity: int):
        """This rank's gathered buffer of the given parity (a torch view)."""
        import hesa_cuda as H
        return H.device_view(self.local + parity * self.y_bytes, self.out_rows, device=self.device)

    def close(self) -> None:
        """Unmap the peers' buffers, then free this rank's (call on every rank,
        after a collective barrier, once no kernel uses them)."""
        import hesa_cuda as H
        for p, b in enumerate(self.base):
            if p != self.rank:
                H.peer_close(b)
        H.peer_free(self.local)
        self.base = []


class TaggedGather:
    """Gathered outputs as tagged 64-bit words (hesa_cuda_qmatvec_gather_tagged).

    Each rank allocates two parities of `out_rows` words and its [step count,
    ticket] pair, and maps every other rank's allocation. Matvecs of a step
    store into every rank (targets); collect() ends the step: it waits until
    this rank's words all carry the step's tag and unpacks them into `out`.
    No barrier kernel, no fence: the data is its own flag.
    """

    def __init__(self, out_rows: int, rank: int, world: int, group=None, device=None):
        import torch
        import torch.distributed as dist
        import hesa_cuda as H
        if not 1 <= world <= 8 or not 0 <= rank < world:
            raise ValueError(f"bad rank {rank} / world {world}")
        self.out_rows, self.rank, self.world = out_rows, rank, world
        self.words = _align(8 * out_rows, 2048) // 8     # parity stride in words: whole units of 256
        self.sync_off = 2 * 8 * self.words
        self.local, handle = H.peer_alloc(self.sync_off + 256)
        handles = [handle]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle, group=group)
        self.base = [self.local if p == rank else H.peer_open(handles[p]) for p in range(world)]
        self.sync = self.local + self.sync_off
        self.out = torch.empty(out_rows, dtype=torch.float32, device=device)
        self.device = device

    def targets(self) -> list[int]:
        """Word 0 of every rank's buffers (parity-major, then rank); a shard
        passes its first row's element index with them."""
        return [b + par * 8 * self.words for par in (0, 1) for b in self.base]

    def collect(self, stream=None):
        """End of a step on this rank: the gathered outputs, in self.out."""
        import hesa_cuda as H
        H.peer_collect(self.local, self.out_rows, self.words, self.out, self.sync, stream=stream)
        return self.out

    def close(self) -> None:
        """Unmap the peers' buffers, then free this rank's (call on every rank,
        after a collective barrier, once no kernel uses them)."""
        import hesa_cuda as H
        for p, b in enumerate(self.base):
            if p != self.rank:
                H.peer_close(b)
        H.peer_free(self.local)
        self.base = []


class GatheredQMatvec:
    """y = scale * W x with W's rows split over the ranks, the all-gather fused
    into the matvec (PeerGather). Every rank calls it with the same x and gets
    the full y (a view valid until the call after next)."""

    def __init__(self, qtype: int, w_rows, n_out: int, k: int, rank: int, world: int, group=None, peers=None,
                 row_offset: int = 0):
        self.qtype, self.n_out, self.k, self.rank, self.world = qtype, n_out, k, rank, world
        self.r0, self.r1 = row_range(n_out, rank, world)
        if w_rows.shape[0] != self.r1 - self.r0:
            raise ValueError(f"rank {rank} holds {w_rows.shape[0]} rows, its shard has {self.r1 - self.r0}")
        self.w = w_rows
        self.own = peers is None
        self.peers = peers or PeerGather(n_out, rank, world, group=group, device=w_rows.device)
        self.row_offset = row_offset
        self.tgt = self.peers.targets(row_offset + self.r0)

    def launch(self, x, scale: float = 1.0, stream=None) -> None:
        """Only the matvec (several may share one barrier)."""
        import hesa_cuda as H
        H.qmatvec_gather(self.qtype, self.w, x, self.tgt, self.world, self.peers.epoch, scale=scale, stream=stream)

    def __call__(self, x, scale: float = 1.0, stream=None):
        par = self.peers.steps & 1
        self.launch(x, scale, stream)
        self.peers.barrier(stream)
        return self.peers.output(par)[self.row_offset:self.row_offset + self.n_out]


class ShardedDecoder:
    """One sequence decoded on `world` GPUs of a node (hesa_cuda_decode_step_sharded).

    Rank r keeps the Q, K, V rows of heads [r*H/world, (r+1)*H/world) (and of
    its kv heads), their KV caches, its balanced row share (row_range) of
    gate|up and of the LM head, and all of Wo and W_down (every rank computes
    their rows itself and keeps the residual locally); the attention output
    and gate|up are gathered into every rank by the kernels that make them, as
    tagged 64-bit words that the consuming kernels wait for (peer stores over
    NVLink, CUDA IPC mappings exchanged through `group`). The logits equal
    the unsharded step's bit for bit.

    full: the unsharded model on this rank's device, laid out as the decode
    step takes it -- a dict with "layers" (dicts of CUDA tensors: wq/wk/wv
    views of one joined Q|K|V allocation, w_gate/w_up of one gate|up
    allocation, wo, w_down, attn_norm, ffn_norm, k_cache, v_cache [ctx, KD]
    fp16), "w_out", "out_norm" and "table" (the device rope table).
    """

    FIELDS = ("a", "gu", "logits", "count")

    def __init__(self, cfg: dict, full: dict, rank: int, world: int, group=None, device=None):
        import torch
        import torch.distributed as dist
        import hesa_cuda as H
        self.cfg, self.rank, self.world = dict(cfg), rank, world
        D, HD, F, V = cfg["d_model"], cfg["head_dim"], cfg["d_ff"], cfg["vocab"]
        NH, NKV = cfg["n_head"], cfg["n_kv_head"]
        if NH % world or NKV % world:
            raise ValueError(f"n_head {NH} and n_kv_head {NKV} must be multiples of world {world}")
        QD, KD = NH * HD, NKV * HD
        qd_r, kd_r = QD // world, KD // world
        f0, f1 = row_range(F, rank, world)
        v0, v1 = row_range(V, rank, world)
        self.rows = dict(f=(f0, f1), v=(v0, v1))
        self.layers = []
        for L in full["layers"]:
            qkv = torch.cat([L["wq"][rank * qd_r:(rank + 1) * qd_r], L["wk"][rank * kd_r:(rank + 1) * kd_r],
                             L["wv"][rank * kd_r:(rank + 1) * kd_r]]).contiguous()
            gu = torch.cat([L["w_gate"][f0:f1], L["w_up"][f0:f1]]).contiguous()
            kc = L["k_cache"][:, rank * kd_r:(rank + 1) * kd_r].contiguous()
            vc = L["v_cache"][:, rank * kd_r:(rank + 1) * kd_r].contiguous()
            self.layers.append(dict(wq=qkv[:qd_r], wk=qkv[qd_r:qd_r + kd_r], wv=qkv[qd_r + kd_r:],
                                    wo=L["wo"].contiguous(), w_gate=gu[:f1 - f0], w_up=gu[f1 - f0:],
                                    w_down=L["w_down"].contiguous(), attn_norm=L["attn_norm"],
                                    ffn_norm=L["ffn_norm"], k_cache=kc, v_cache=vc, _keep=(qkv, gu)))
        self.w_out = full["w_out"][v0:v1].contiguous()
        self.out_norm, self.table = full["out_norm"], full["table"]
        self.model = H.Model(cfg["n_layer"], D, NH, NKV, HD, F, V, cfg["ctx"], cfg["rms_eps"], cfg["rope_base"],
                             cfg["qtype"])
        self.arr = H.make_layers(self.layers)
        self.ws = H.decode_workspace(self.model, device)
        # one peer allocation per rank: tagged words (8 bytes) of a | gate,up |
        # logits, then the token counter; tagged vectors hold whole units of
        # 256 words (the up half of gate|up starts at element F, a multiple of
        # 256)
        sizes = dict(a=8 * _align(QD), gu=16 * _align(F), logits=8 * _align(V), count=4)
        self.off, total = {}, 0
        for name in self.FIELDS:
            self.off[name] = total
            total += _align(sizes[name])
        self.local, handle = H.peer_alloc(total)
        handles = [handle]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle, group=group)
        self.base = [self.local if p == rank else H.peer_open(handles[p]) for p in range(world)]
        self.device = device
        self.shard = H.Shard(rank, world, *[self._ptrs(n) for n in ("a", "gu", "logits")],
                             self.local + self.off["count"])
        self.out = torch.empty(V, dtype=torch.float32, device=device)

    def _ptrs(self, name):
        import ctypes
        arr = (ctypes.c_void_p * self.world)(*[b + self.off[name] for b in self.base])
        setattr(self, "_arr_" + name, arr)   # keep it alive with the struct
        return arr

    def logits(self):
        """All the logits of the last step (this rank's device memory)."""
        return self.out

    def step(self, x_embed, pos_dev, stream=None) -> None:
        """One token: every rank calls it with the same embedding and position."""
        import hesa_cuda as H
        H.decode_step_sharded(self.model, self.shard, self.arr, self.out_norm, self.w_out, self.table, x_embed,
                              pos_dev, self.out, self.ws, stream=stream)

    def close(self) -> None:
        """Unmap the peers' buffers, then free this rank's (every rank, after a
        collective barrier, once no kernel uses them)."""
        import hesa_cuda as H
        for p, b in enumerate(self.base):
            if p != self.rank:
                H.peer_close(b)
        H.peer_free(self.local)
        self.base = []
