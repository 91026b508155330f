"""Python face of the INT8 group-64 linear library, named like the reference.

The reference launchers (src/model_cuda_v2_shared.cu, declared in
include/model.h:62-64) take raw device pointers and sizes:

    matmul_int8(xout, x, w_q, w_s, n, d, group_size)
    matmul_dp4a(xout, x_q, x_s, w_q, w_s, n, d, group_size)
    quantize_activation(xq, xs, x, n)

These functions keep those names, argument orders and meanings, accept CUDA
torch tensors (or raw device pointers as ints) and forward to the C ABI on the
current torch stream.  Unlike the reference, which checks nothing, a failing
call raises MliError.  torch is used only as a device-memory container.
"""
from __future__ import annotations

import ctypes

from ._lib import GemvOp, check, lib

__all__ = [
    "matmul", "matmul_int8", "matmul_dp4a", "quantize_activation", "matmul_dp4a_fused",
    "quantize_activation_rows", "gemm_w8a8", "gemm_w8a8_cuda_core", "gemm_workspace_bytes",
    "quantize_weights", "group_dots",
    "device_error", "set_pdl", "copy_from_ptr", "GemvChain", "DECODE_LAYER_WAITS",
]


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor (device memory)")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def matmul(xout, x, w, n: int, d: int, stream=None):
    """fp32 GEMV, xout[d] = w[d][n] @ x[n] (reference :10-25, the classifier's launcher)."""
    check(lib().mli_gemv_f32(_ptr(xout), _ptr(x), _ptr(w), n, d, _stream(stream)), "matmul")


def matmul_int8(xout, x, w_q, w_s, n: int, d: int, group_size: int = 64, stream=None):
    """W8A32 GEMV, xout[d] = dequant(w_q, w_s)[d][n] @ x[n] (reference :36-69)."""
    check(lib().mli_gemv_w8a32(_ptr(xout), _ptr(x), _ptr(w_q), _ptr(w_s), n, d, group_size,
                               _stream(stream)), "matmul_int8")


def quantize_activation(xq, xs, x, n: int, stream=None):
    """Per-token int8 quantisation of x[n] (reference :429-460)."""
    check(lib().mli_quantize_activation(_ptr(xq), _ptr(xs), _ptr(x), n, _stream(stream)),
          "quantize_activation")


def matmul_dp4a(xout, x_q, x_s, w_q, w_s, n: int, d: int, group_size: int = 64, stream=None):
    """W8A8 GEMV from an already-quantised activation (reference :462-509)."""
    check(lib().mli_gemv_w8a8(_ptr(xout), _ptr(x_q), _ptr(x_s), _ptr(w_q), _ptr(w_s), n, d,
                              group_size, _stream(stream)), "matmul_dp4a")


def matmul_dp4a_fused(xout, x, w_q, w_s, n: int, d: int, group_size: int = 64,
                      xq_out=None, xs_out=None, stream=None):
    """W8A8 GEMV with the activation quantiser fused in (one launch)."""
    check(lib().mli_gemv_w8a8_fused(_ptr(xout), _ptr(xq_out), _ptr(xs_out), _ptr(x), _ptr(w_q),
                                    _ptr(w_s), n, d, group_size, _stream(stream)),
          "matmul_dp4a_fused")


def quantize_activation_rows(xq, xs, x, m: int, n: int, stream=None):
    check(lib().mli_quantize_activation_rows(_ptr(xq), _ptr(xs), _ptr(x), m, n, _stream(stream)),
          "quantize_activation_rows")


def gemm_workspace_bytes(m: int, n: int, d: int) -> int:
    return int(lib().mli_gemm_w8a8_workspace_bytes(m, n, d))


def gemm_w8a8(y, xq, xs, w_q, w_s, m: int, n: int, d: int, group_size: int = 64, workspace=None,
              stream=None):
    """Batched W8A8 for m tokens: y[m][d].  `workspace`: a zero-initialised
    uint8 CUDA tensor of gemm_workspace_bytes(m, n, d) bytes (optional)."""
    ws_ptr, ws_bytes = (None, 0) if workspace is None else (_ptr(workspace), workspace.numel())
    check(lib().mli_gemm_w8a8(_ptr(y), _ptr(xq), _ptr(xs), _ptr(w_q), _ptr(w_s), m, n, d,
                              group_size, ws_ptr, ws_bytes, _stream(stream)), "gemm_w8a8")


def gemm_w8a8_group(items, m: int, group_size: int = 64, stream=None):
    """Several independent batched W8A8 GEMMs of m tokens in one launch.
    items: (y, xq, xs, w_q, w_s, n, d) tuples, at most 8."""
    from ._lib import GemmOp

    arr = (GemmOp * len(items))()
    for i, (y, xq, xs, w_q, w_s, n, d) in enumerate(items):
        arr[i] = GemmOp(_ptr(y), _ptr(xq), _ptr(xs), _ptr(w_q), _ptr(w_s), n, d)
    check(lib().mli_gemm_w8a8_group(arr, len(items), m, group_size, _stream(stream)), "gemm_w8a8_group")


def gemm_group_plan(items, m: int) -> dict:
    """The persistent plan mli_gemm_w8a8_group would take for these items
    (same tuples as gemm_w8a8_group; nothing is launched)."""
    from ._lib import GemmOp

    arr = (GemmOp * len(items))()
    for i, (y, xq, xs, w_q, w_s, n, d) in enumerate(items):
        arr[i] = GemmOp(_ptr(y), _ptr(xq), _ptr(xs), _ptr(w_q), _ptr(w_s), n, d)
    out = (ctypes.c_int * 5)()
    check(lib().mli_debug_plan_gemm_group(arr, len(items), m, out), "debug_plan_gemm_group")
    return {"persistent": bool(out[0]), "ctas": out[1], "tiles": out[2], "busiest": out[3], "total": out[4]}


def set_gemm_persistent(enabled: bool) -> None:
    """Batched W8A8 above 64 tokens: let well-balanced problems run on the
    persistent whole-tile kernel (default), or always take the split-K ones."""
    from ._lib import MLI_LAUNCH_NO_PERSISTENT
    flags = lib().mli_get_launch_flags()
    flags = (flags & ~MLI_LAUNCH_NO_PERSISTENT) if enabled else (flags | MLI_LAUNCH_NO_PERSISTENT)
    lib().mli_set_launch_flags(flags)


def gemm_w8a8_cuda_core(y, xq, xs, w_q, w_s, m: int, n: int, d: int, group_size: int = 64, stream=None):
    check(lib().mli_gemm_w8a8_cuda_core(_ptr(y), _ptr(xq), _ptr(xs), _ptr(w_q), _ptr(w_s), m, n, d,
                                        group_size, _stream(stream)), "gemm_w8a8_cuda_core")


def quantize_weights(w_q, w_s, w, rows: int, cols: int, group_size: int = 64, stream=None):
    """Group-wise weight quantisation (scripts/quantize_int8_group.py:55-71)."""
    check(lib().mli_quantize_weights(_ptr(w_q), _ptr(w_s), _ptr(w), rows, cols, group_size,
                                     _stream(stream)), "quantize_weights")


def group_dots(out, xq, w_q, n: int, d: int, group_size: int = 64, stream=None):
    check(lib().mli_debug_group_dots(_ptr(out), _ptr(xq), _ptr(w_q), n, d, group_size,
                                     _stream(stream)), "group_dots")


def device_error() -> int:
    code = ctypes.c_uint(0)
    lib().mli_device_error(ctypes.byref(code))
    return int(code.value)


def copy_from_ptr(dst, src_ptr: int, nbytes: int) -> None:
    """Synchronous device-to-device copy from a raw device pointer (e.g. a peer
    block of the row-sharded layer) into the CUDA tensor `dst`."""
    lib()
    for name in ("libcudart.so.12", "libcudart.so"):
        try:
            rt = ctypes.CDLL(name)
            break
        except OSError:
            rt = None
    if rt is None:
        raise OSError("libcudart not found")
    rc = rt.cudaMemcpy(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src_ptr), ctypes.c_size_t(nbytes), 3)
    if rc != 0:
        raise RuntimeError(f"cudaMemcpy failed: {rc}")


def set_pdl(enabled: bool) -> None:
    flags = lib().mli_get_launch_flags()
    flags = (flags | 1) if enabled else (flags & ~1)
    lib().mli_set_launch_flags(flags)


def set_gemm_clusters(enabled: bool) -> None:
    """Batched W8A8 split-K: sum the K splits of a tile inside a thread-block
    cluster (default), or through the caller's workspace."""
    from ._lib import MLI_LAUNCH_NO_CLUSTER
    flags = lib().mli_get_launch_flags()
    flags = (flags & ~MLI_LAUNCH_NO_CLUSTER) if enabled else (flags | MLI_LAUNCH_NO_CLUSTER)
    lib().mli_set_launch_flags(flags)


# Waits of a decode layer's GEMVs q, k, v, o, gate, up, down at chain index
# b + 0..6, relative to b: o after q/k/v (attention), gate/up after o (residual
# + norm), down after gate/up (SwiGLU); the next layer's q/k/v wait for down.
DECODE_LAYER_WAITS = (0, 0, 0, 3, 4, 4, 6)
_FORMS = {"w8a32": 0, "w8a8": 1, "w8a8_fused": 2}
_EPILOGUES = {"store": 0, "add": 1, "swiglu": 2}


class GemvChain:
    """A chain of batch-1 GEMVs run as one persistent launch (mli_chain_*).

    `ops` is a sequence of dicts with keys form ("w8a32", "w8a8" or
    "w8a8_fused"), y, w_q, w_s, n, d, wait and x (or xq and xs for "w8a8");
    tensors or raw device pointers.  Op i reads its activation only once ops
    [0, wait) have finished.  Each op's y is bit-identical to the single call
    (matmul_int8 / matmul_dp4a / matmul_dp4a_fused).  Optional "epilogue":
    "store" (default), "add" (y += the op's rows: the residual add), or
    "swiglu" (this op is the gate and the NEXT op the up projection, same n, d,
    x and wait; y = silu(gate) * up; the next op's y may be None).  Optional
    "norm_w": the activation is RMSNorm(x) * norm_w (the reference's
    rmsnorm_cuda), computed in the op's prologue.  An op reading the y of an
    earlier op takes that op's rows of the same launch; an "add" op adds into
    the latest earlier op's output of the same y.  The buffers must outlive
    the chain; the chain keeps references to the tensors given.

    Row-sharded chains (mli_chain_create_sharded): every op dict may carry
    "row_offset" and "d_total" (default 0 and d): the op computes rows
    [row_offset, row_offset + d) of a GEMV of d_total rows, its y pointing at
    the first of them, and an op whose x is the whole vector (the producer's
    y - row_offset) reads every rank's rows.  `world` > 1 makes the chain
    share its rows over NVLink: call export() on every rank, exchange the
    handles, then set_peers(handles, rank) before the first run.
    """

    def __init__(self, ops, group_size: int = 64, world: int = 1):
        arr = (GemvOp * len(ops))()
        self._keep = []
        for i, o in enumerate(ops):
            e = arr[i]
            e.form = _FORMS[o["form"]]
            e.n, e.d, e.group_size, e.wait = o["n"], o["d"], group_size, o.get("wait", 0)
            e.epilogue = _EPILOGUES[o.get("epilogue", "store")]
            for key in ("y", "x", "xq", "xs", "w_q", "w_s", "norm_w"):
                t = o.get(key)
                setattr(e, key, _ptr(t))
                if t is not None and not isinstance(t, int):
                    self._keep.append(t)
        self.count = len(ops)
        self.world = world
        self.d_total = [o.get("d_total", o["d"]) for o in ops]
        self._peers = []
        self._h = ctypes.c_void_p()
        sharded = world > 1 or any("row_offset" in o or "d_total" in o for o in ops)
        if sharded:
            roff = (ctypes.c_int * len(ops))(*[o.get("row_offset", 0) for o in ops])
            dtot = (ctypes.c_int * len(ops))(*self.d_total)
            check(lib().mli_chain_create_sharded(arr, roff, dtot, len(ops), world, ctypes.byref(self._h)),
                  "mli_chain_create_sharded")
        else:
            check(lib().mli_chain_create(arr, len(ops), ctypes.byref(self._h)), "mli_chain_create")

    def export(self) -> bytes:
        """The 64-byte CUDA IPC handle of this rank's mirror block."""
        buf = ctypes.create_string_buffer(64)
        check(lib().mli_chain_export(self._h, buf), "mli_chain_export")
        return buf.raw

    def set_peers(self, handles, rank: int) -> None:
        """handles[r]: rank r's export(); this rank's own entry is not opened."""
        ptrs = (ctypes.c_void_p * self.world)()
        for r, h in enumerate(handles):
            if r == rank:
                continue
            p = ctypes.c_void_p()
            check(lib().mli_peer_open(h, ctypes.byref(p)), "mli_peer_open")
            self._peers.append(p)
            ptrs[r] = p.value
        check(lib().mli_chain_set_peers(self._h, ptrs, rank), "mli_chain_set_peers")

    def set_peer_pointers(self, ptrs, rank: int) -> None:
        """Every rank's mirror block as device pointers already mapped in this
        process (ptrs[rank] is ignored): for frameworks that share memory
        their own way."""
        arr = (ctypes.c_void_p * self.world)(*[0 if r == rank else int(p) for r, p in enumerate(ptrs)])
        check(lib().mli_chain_set_peers(self._h, arr, rank), "mli_chain_set_peers")

    def rows(self, op: int):
        """(whole rows of op `op` from the last run as a numpy float32 array,
        True when every row carries that run's tag); synchronous."""
        import numpy as np

        out = np.empty(self.d_total[op], np.float32)
        ok = ctypes.c_int(0)
        check(lib().mli_chain_rows(self._h, op, out.ctypes.data, ctypes.byref(ok)), "mli_chain_rows")
        return out, bool(ok.value)

    def run(self, stream=None):
        check(lib().mli_chain_run(self._h, _stream(stream)), "mli_chain_run")

    def close(self):
        if self._h is not None and self._h.value:
            lib().mli_chain_destroy(self._h)
        self._h = None
        for p in self._peers:
            lib().mli_peer_close(p)
        self._peers = []
        self._keep = []

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
