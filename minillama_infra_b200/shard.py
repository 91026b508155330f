"""Row-sharded INT8 group-64 linear layer across the GPUs of one node.

The 128256x2048 tied-embedding classifier of Llama-3.2-1B (src/model_cuda_v2_shared.cu:418,
:564 in the reference, where it is a single-GPU fp32 matmul) and the FFN gate/up/down
projections shard naturally by output rows: every row is an independent full-K dot, so no
reduction crosses GPUs.  Rank r owns rows [r*chunk, min(d, (r+1)*chunk)) with
chunk = ceil(d / world); after the local GEMV the fp32 outputs are all-gathered so every
rank holds the full vector.  Because the GEMV's per-row arithmetic depends only on n, the
gathered logits are bit-identical to the single-GPU result for any world size, and so is
their argmax.

One process per GPU; torch.distributed carries the collective (NCCL on GPUs, gloo in the
CPU tests).  `compute` is pluggable so the same host logic runs over the CUDA kernels or,
in the CPU tests, over the oracle.
"""
from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class RowShard:
    d: int          # total rows
    world: int
    rank: int

    @property
    def chunk(self) -> int:
        return math.ceil(self.d / self.world)

    @property
    def r0(self) -> int:
        return min(self.d, self.rank * self.chunk)

    @property
    def r1(self) -> int:
        return min(self.d, (self.rank + 1) * self.chunk)

    @property
    def rows(self) -> int:
        return self.r1 - self.r0


def row_shard(d: int, world: int, rank: int) -> RowShard:
    if world <= 0 or not (0 <= rank < world) or d <= 0:
        raise ValueError(f"bad shard request d={d} world={world} rank={rank}")
    return RowShard(d, world, rank)


class ShardedLinear:
    """One rank's share of a row-sharded INT8 group-64 linear layer.

    w_q / w_s hold only this rank's rows (int8 [rows][n], fp32 [rows][n/64]).
    forward(x) computes the local rows into a padded chunk buffer and all-gathers the
    chunks into `full`, whose first d entries are the layer's output in row order.
    """

    def __init__(self, w_q, w_s, d: int, n: int, rank: int, world: int, form: str = "w8a32",
                 group=None, compute=None, device=None):
        import torch

        self.shard = row_shard(d, world, rank)
        if w_q.shape[0] != self.shard.rows or w_q.shape[1] != n:
            raise ValueError(f"weight shard {tuple(w_q.shape)} != ({self.shard.rows}, {n})")
        if form not in ("w8a32", "w8a8"):
            raise ValueError(f"unknown form {form}")
        self.w_q, self.w_s, self.d, self.n, self.form = w_q, w_s, d, n, form
        self.group = group
        self.device = w_q.device if device is None else device
        self.local = torch.zeros(self.shard.chunk, dtype=torch.float32, device=self.device)
        self.full = torch.zeros(self.shard.chunk * world, dtype=torch.float32, device=self.device)
        self.compute = compute if compute is not None else self._compute_cuda

    def _compute_cuda(self, y, x):
        from . import ops

        if self.shard.rows == 0:
            return
        if self.form == "w8a32":
            ops.matmul_int8(y, x, self.w_q, self.w_s, self.n, self.shard.rows, 64)
        else:
            ops.matmul_dp4a_fused(y, x, self.w_q, self.w_s, self.n, self.shard.rows, 64)

    def forward(self, x):
        import torch.distributed as dist

        self.compute(self.local[: self.shard.rows], x)
        if dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(self.full, self.local, group=self.group)
        else:
            parts = list(self.full.view(self.shard.world, self.shard.chunk).unbind(0))
            dist.all_gather(parts, self.local, group=self.group)
        return self.full[: self.d]


def rowshard_tag(step: int) -> int:
    """Tag of the words a row-sharded step writes (mli_rowshard_block_bytes)."""
    return step % 4095 + 1


def read_tagged_logits(ptr: int, d: int, half: int, step: int):
    """The fp32 logits of step `step` from a peer block's logits words at
    device address `ptr` (offset 256 of the block), checking that every word
    carries that step's tag.  Call it once every rank has finished the step."""
    import numpy as np
    import torch

    from . import ops

    raw = torch.empty(d, dtype=torch.int64, device=torch.cuda.current_device())
    torch.cuda.synchronize()
    ops.copy_from_ptr(raw, ptr + half * d * 8, d * 8)
    words = raw.cpu().numpy().view(np.uint32).reshape(d, 2)
    if not np.all(words[:, 1] == rowshard_tag(step)):
        bad = int(np.count_nonzero(words[:, 1] != rowshard_tag(step)))
        raise RuntimeError(f"{bad} of {d} logits words do not carry step {step}'s tag")
    return words[:, 0].copy().view(np.float32)


class PeerShardedLinear:
    """Row-sharded layer whose all-gather is fused into the GEMV.

    Every rank allocates one peer block (CUDA IPC, no multicast; layout in
    include/mli_gemv.h, mli_rowshard_block_bytes):
        [128, 132) uint32 step counter (local)
        [192, 196) uint32 finished-CTA count of a fused step (local)
        [256, ...) logits words uint64 [2][d] ({fp32 value, step tag}; the half
                   is the step's parity), then the CTAs' tagged (max, first
                   index) partial words
    and opens every other rank's block.  A step is one launch on the current
    stream, mli_gemv_rowshard_argmax: this rank's rows, tagged with the step,
    stored into every rank's logits, each CTA's partial word into every rank's
    block; the launch's last CTA polls (bounded) all ranks' partial words of
    this step, takes the argmax and advances the step.  Nothing waits for a
    fence: each word tells by its tag whether it belongs to this step.
    (forward(fused=False) runs the same as two launches, mli_gemv_rowshard +
    mli_rowshard_wait_argmax.)  The handles travel through torch.distributed
    (any backend); no collective runs on the data path.  world == 1 needs no
    process group (the single GPU then gets the fused GEMV + argmax).
    """

    HEADER = 256

    def __init__(self, w_q, w_s, d: int, n: int, rank: int, world: int, form: str = "w8a32",
                 group=None, timeout_us: int = 2_000_000):
        import ctypes

        import torch
        import torch.distributed as dist

        from ._lib import check, lib

        self.shard = row_shard(d, world, rank)
        if form not in ("w8a32", "w8a8"):
            raise ValueError(f"unknown form {form}")
        if world > 8:
            raise ValueError("at most 8 ranks")
        self.w_q, self.w_s, self.d, self.n, self.rank, self.world = w_q, w_s, d, n, rank, world
        self.form_code = 0 if form == "w8a32" else 2
        self.timeout_us = timeout_us
        self.lib = lib()
        nbytes = self.lib.mli_rowshard_block_bytes(d)
        self._own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        check(self.lib.mli_peer_alloc(nbytes, ctypes.byref(self._own), handle), "mli_peer_alloc")
        handles = [handle.raw]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle.raw, group=group)
        self._opened = []
        bases = []
        for p in range(world):
            if p == rank:
                bases.append(self._own.value)
                continue
            ptr = ctypes.c_void_p()
            check(self.lib.mli_peer_open(handles[p], ctypes.byref(ptr)), "mli_peer_open")
            self._opened.append(ptr.value)
            bases.append(ptr.value)
        P = ctypes.c_void_p
        self._peer_logits = (P * world)(*[b + self.HEADER for b in bases])
        self._shard_rows = (ctypes.c_int * world)(*[row_shard(d, world, r).rows for r in range(world)])
        self.base = self._own.value
        self.out = torch.zeros((), dtype=torch.int64, device=w_q.device)
        self.steps = 0
        self.group = group
        if world > 1:
            dist.barrier(group=group)  # every rank has opened every block before any step

    def logits(self, half: int):
        """Device address of this rank's logits words of one half (0 or 1)."""
        return self.base + self.HEADER + half * self.d * 8

    def read_logits(self, step: int):
        """fp32 logits of step `step` (0-based) from this rank's block; every
        rank must have finished that step."""
        return read_tagged_logits(self.base + self.HEADER, self.d, step & 1, step)

    def forward(self, x, stream=None, fused: bool = True, out=None):
        """One step: this rank's rows to every rank, then the argmax into
        `out` (an int64 device scalar; default self.out) -- one launch (fused)
        or the GEMV and the wait kernel.  Returns the tensor written."""
        import torch

        from ._lib import check

        st = torch.cuda.current_stream().cuda_stream if stream is None else stream
        if out is None:
            out = self.out
        elif out.dtype != torch.int64 or out.numel() != 1 or out.device != self.out.device:
            raise ValueError("out must be one int64 element on this rank's device")
        if fused:
            check(self.lib.mli_gemv_rowshard_argmax(
                self.form_code, self._peer_logits, self.base, x.data_ptr(), self.w_q.data_ptr(),
                self.w_s.data_ptr(), self.n, self.shard.rows, self.shard.r0, self.d, self.rank, self.world, 64,
                self._shard_rows, out.data_ptr(), self.timeout_us, st), "mli_gemv_rowshard_argmax")
        else:
            check(self.lib.mli_gemv_rowshard(self.form_code, self._peer_logits, self.base + 128, x.data_ptr(),
                                             self.w_q.data_ptr(), self.w_s.data_ptr(), self.n, self.shard.rows,
                                             self.shard.r0, self.d, self.rank, self.world, 64, st),
                  "mli_gemv_rowshard")
            check(self.lib.mli_rowshard_wait_argmax(self.form_code, self.n, self.base + self.HEADER,
                                                    self.base + 128, self._shard_rows, self.world, self.d,
                                                    out.data_ptr(), self.timeout_us, st),
                  "mli_rowshard_wait_argmax")
        self.steps += 1
        return out

    def close(self):
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        for p in self._opened:
            self.lib.mli_peer_close(p)
        self._opened = []
        if self.world > 1:
            dist.barrier(group=self.group)
        if self._own.value:
            self.lib.mli_peer_free(self._own.value)
            self._own.value = None


class ShardedFFN:
    """One rank's share of a row-sharded Llama FFN block: gate/up/down.

    The reference runs the block on one GPU (src/model_cuda_v2_shared.cu:408-412 W8A32,
    :551-558 W8A8): hb = gate(xb), hb2 = up(xb), hb = silu(hb) * hb2, xb = down(hb).
    Sharded over `world` ranks by output rows:

      1. gate/up rows [r0, r1) of the hidden dimension (hidden / world rows each):
         hb_local = silu(gate_local x) * (up_local x), in ONE launch (a two-op chain whose
         SwiGLU epilogue streams both matrices' rows together);
      2. all-gather hb (hidden fp32) so every rank holds the whole vector;
      3. down rows [r0', r1') of the model dimension (dim / world rows, K = hidden);
      4. all-gather xb (dim fp32).

    Every row is a full-K dot whose arithmetic depends only on K, so the gathered hb and xb
    are bit-identical to the single-GPU block for any world size.  `gate_q` ... `down_s` are
    this rank's rows only.  `form`: "w8a32" or "w8a8" (activation quantisation fused into
    each GEMV, as mli_gemv_w8a8_fused).  `compute_gateup(hb_local, x)` and
    `compute_down(y_local, hb)` default to the CUDA kernels; the CPU tests pass the oracle.
    """

    def __init__(self, gate_q, gate_s, up_q, up_s, down_q, down_s, dim: int, hidden: int,
                 rank: int, world: int, form: str = "w8a32", group=None,
                 compute_gateup=None, compute_down=None, device=None):
        import torch

        if form not in ("w8a32", "w8a8"):
            raise ValueError(f"unknown form {form}")
        self.hs = row_shard(hidden, world, rank)   # gate/up rows
        self.ds = row_shard(dim, world, rank)      # down rows
        for name, t, rows, cols in (("gate", gate_q, self.hs.rows, dim), ("up", up_q, self.hs.rows, dim),
                                    ("down", down_q, self.ds.rows, hidden)):
            if tuple(t.shape) != (rows, cols):
                raise ValueError(f"{name} shard {tuple(t.shape)} != ({rows}, {cols})")
        self.gate_q, self.gate_s, self.up_q, self.up_s = gate_q, gate_s, up_q, up_s
        self.down_q, self.down_s = down_q, down_s
        self.dim, self.hidden, self.world, self.form, self.group = dim, hidden, world, form, group
        self.device = gate_q.device if device is None else device
        f32 = dict(dtype=torch.float32, device=self.device)
        self.hb_local = torch.zeros(self.hs.chunk, **f32)
        self.hb_full = torch.zeros(self.hs.chunk * world, **f32)
        self.xb_local = torch.zeros(self.ds.chunk, **f32)
        self.xb_full = torch.zeros(self.ds.chunk * world, **f32)
        self._x = None
        self._chain = None
        self.compute_gateup = compute_gateup if compute_gateup is not None else self._gateup_cuda
        self.compute_down = compute_down if compute_down is not None else self._down_cuda

    def _gateup_cuda(self, hb_local, x):
        from . import ops

        if self.hs.rows == 0:
            return
        if self._chain is None or self._x is not x:
            if self._chain is not None:
                self._chain.close()
            form = "w8a32" if self.form == "w8a32" else "w8a8_fused"
            rows = self.hs.rows
            self._chain = ops.GemvChain([
                dict(form=form, n=self.dim, d=rows, wait=0, x=x, y=hb_local, w_q=self.gate_q, w_s=self.gate_s,
                     epilogue="swiglu"),
                dict(form=form, n=self.dim, d=rows, wait=0, x=x, y=None, w_q=self.up_q, w_s=self.up_s),
            ])
            self._x = x
        self._chain.run()

    def _down_cuda(self, y_local, hb):
        from . import ops

        if self.ds.rows == 0:
            return
        if self.form == "w8a32":
            ops.matmul_int8(y_local, hb, self.down_q, self.down_s, self.hidden, self.ds.rows, 64)
        else:
            ops.matmul_dp4a_fused(y_local, hb, self.down_q, self.down_s, self.hidden, self.ds.rows, 64)

    def _gather(self, full, local, shard):
        import torch.distributed as dist

        if self.world == 1:
            full.copy_(local)
        elif dist.get_backend(self.group) == "nccl":
            dist.all_gather_into_tensor(full, local, group=self.group)
        else:
            parts = list(full.view(self.world, shard.chunk).unbind(0))
            dist.all_gather(parts, local, group=self.group)

    def forward(self, x):
        """xb = down(silu(gate x) * (up x)) over all ranks; returns the dim-vector."""
        self.compute_gateup(self.hb_local[: self.hs.rows], x)
        self._gather(self.hb_full, self.hb_local, self.hs)
        self.compute_down(self.xb_local[: self.ds.rows], self.hb_full[: self.hidden])
        self._gather(self.xb_full, self.xb_local, self.ds)
        return self.xb_full[: self.dim]

    def hidden_vector(self):
        """The gathered silu(gate x) * (up x) of the last forward."""
        return self.hb_full[: self.hidden]

    def close(self):
        if self._chain is not None:
            self._chain.close()
            self._chain = None


class ChainShardedFFN:
    """A stack of row-sharded Llama FFN blocks as ONE chained launch per step
    on every rank, with the exchanges between ranks inside the kernel.

    Per layer l (the reference's block, src/model_cuda_v2_shared.cu:408-412
    W8A32, :551-558 W8A8): hb = silu(gate x) * (up x), x' = down hb, and the
    next layer reads x'.  Rank r computes gate/up rows [r0, r1) of the hidden
    dimension (one SwiGLU pair of the chain) and down rows [r0', r1') of the
    model dimension.  Each rank stores every row it computes, tagged with the
    launch, into every rank's copy of the vector over NVLink
    (mli_chain_create_sharded), and the next op of every rank starts as soon
    as the tagged rows it reads have arrived: no NCCL call, no host
    synchronisation, no fence.  Every row is a full-K dot whose arithmetic
    depends only on K, so every hb and x' is bit-identical to the same chain
    on one GPU for any world size.

    `layers`: this rank's shards, (gate_q, gate_s, up_q, up_s, down_q, down_s)
    per layer; `x0`: the first layer's input (dim fp32, read at launch);
    `exchange(bytes) -> list of bytes`: every rank's 64-byte handle, in rank
    order (e.g. torch.distributed.all_gather_object); without it (world > 1)
    the caller sets the peers itself (self.chain.set_peers /
    set_peer_pointers) before the first run.  Every rank must own
    rows of both dimensions.  Close it on every rank only after all ranks'
    last runs have finished (a barrier), since peers write into this rank's
    buffers.
    """

    def __init__(self, layers, x0, dim: int, hidden: int, rank: int, world: int, form: str = "w8a32",
                 exchange=None):
        import torch

        from . import ops

        if form not in ("w8a32", "w8a8"):
            raise ValueError(f"unknown form {form}")
        self.hs = row_shard(hidden, world, rank)
        self.ds = row_shard(dim, world, rank)
        if self.hs.rows == 0 or self.ds.rows == 0:
            raise ValueError("every rank must own rows of both dimensions")
        self.dim, self.hidden, self.rank, self.world, self.form = dim, hidden, rank, world, form
        dev = x0.device
        self.hb = torch.zeros(self.hs.chunk * world, dtype=torch.float32, device=dev)
        self.xb = torch.zeros(self.ds.chunk * world, dtype=torch.float32, device=dev)
        self.x0 = x0
        f = "w8a32" if form == "w8a32" else "w8a8_fused"
        chain_ops = []
        for l, (gq, gs, uq, us, dq, ds_) in enumerate(layers):
            b = 3 * l
            x = x0 if l == 0 else self.xb
            common = dict(form=f, n=dim, d=self.hs.rows, wait=b, x=x, row_offset=self.hs.r0, d_total=hidden)
            chain_ops.append(dict(common, y=self.hb[self.hs.r0:], w_q=gq, w_s=gs, epilogue="swiglu"))
            chain_ops.append(dict(common, y=None, w_q=uq, w_s=us))
            chain_ops.append(dict(form=f, n=hidden, d=self.ds.rows, wait=b + 2, x=self.hb, y=self.xb[self.ds.r0:],
                                  w_q=dq, w_s=ds_, row_offset=self.ds.r0, d_total=dim))
        self.layers = len(layers)
        self.chain = ops.GemvChain(chain_ops, world=world)
        if world > 1 and exchange is not None:
            self.chain.set_peers(exchange(self.chain.export()), rank)

    def run(self, stream=None):
        self.chain.run(stream)

    def hidden_rows(self, layer: int):
        """(hb of `layer` from the last run, every row tagged)."""
        return self.chain.rows(3 * layer)

    def output_rows(self, layer: int = -1):
        """(x' of `layer` (default: the last) from the last run, every row tagged)."""
        l = layer % self.layers
        return self.chain.rows(3 * l + 2)

    def close(self):
        if self.chain is not None:
            self.chain.close()
            self.chain = None
