"""Thin object layer over the C ABI: a device context and uploaded q4nx weights.

Device buffers may be torch tensors (any object with ``data_ptr()``) or raw
integer addresses; torch is used only as plumbing (allocation, streams).
"""

from __future__ import annotations

import ctypes
import weakref

import numpy as np

from . import _lib
from ._lib import check


def _ptr(t) -> int:
    if t is None:
        return 0
    if isinstance(t, int):
        return t
    return int(t.data_ptr())


_char_from_buffer = ctypes.c_char.from_buffer


def _np_addr(a: np.ndarray) -> int:
    """Address of a C-contiguous host array's first byte (a writable array's
    through the buffer protocol, which costs a fraction of ``a.ctypes``)."""
    if a.flags.writeable and a.size:
        return ctypes.addressof(_char_from_buffer(a))
    return a.ctypes.data


def _stream_for(stream, *tensors) -> int:
    """The stream to launch on: an explicit one, else the current torch stream of
    the first torch tensor argument (so launches are ordered after the torch
    copies/allocations that produced the buffers), else 0 = the context stream."""
    if stream is not None:
        return int(stream)
    for t in tensors:
        if t is not None and hasattr(t, "device") and getattr(t, "is_cuda", False):
            import torch
            h = int(torch.cuda.current_stream(t.device).cuda_stream)
            # torch reports the legacy default stream as 0, which the C ABI
            # reads as "the context's own stream": pass cudaStreamLegacy instead.
            return h if h != 0 else CUDA_STREAM_LEGACY
    return 0


CUDA_STREAM_LEGACY = 1   # cudaStreamLegacy


class Context:
    """One CUDA context slot of the library: a stream, SM count and scratch."""

    def __init__(self, device: int = 0):
        self.lib = _lib.load()
        h = ctypes.c_void_p()
        check(self.lib.rc_init(int(device), ctypes.byref(h)), "rc_init")
        self.handle = h
        self.device = int(device)
        s = ctypes.c_void_p()
        check(self.lib.rc_stream(h, ctypes.byref(s)))
        self.stream = s.value or 0
        n = ctypes.c_int()
        check(self.lib.rc_sm_count(h, ctypes.byref(n)))
        self.sm_count = n.value
        # Objects created on this context; they are released before it is.
        self._children = weakref.WeakSet()

    def _adopt(self, obj) -> None:
        self._children.add(obj)

    def sync(self) -> None:
        check(self.lib.rc_sync(self.handle), "rc_sync")

    def close(self) -> None:
        if self.handle:
            for child in list(self._children):
                child.release()
            self.lib.rc_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def upload_q4nx(self, packed, n: int, k: int, gate_up: bool = False) -> "Q4nxWeight":
        return Q4nxWeight(self, packed, n, k, gate_up=gate_up)

    def upload_bfp16(self, packed, n: int, k: int) -> "Bfp16Weight":
        """A bfp16ebs8 matrix from the reference's ``pack_bfp16_gemv`` bytes (N*K*9/8)."""
        return Bfp16Weight(self, packed, n, k)

    def quantize_q4nx(self, w_dev, packed_dev, n: int, k: int, stream: int | None = None) -> None:
        """f32 [n, k] device weights -> pack_gemv bytes on the device (synchronous)."""
        check(self.lib.rc_quantize_q4nx(self.handle, ctypes.c_void_p(_ptr(w_dev)), int(n), int(k),
                                        ctypes.c_void_p(_ptr(packed_dev)),
                                        ctypes.c_void_p(_stream_for(stream, w_dev, packed_dev))),
              "rc_quantize_q4nx")


def sample_tokens(ctx: "Context", logits_dev, u_dev, out_dev, top_k: int = 50, top_p: float = 0.9,
                  temperature: float = 1.0, presence_penalty: float = 0.0, seen_dev=None, seen_off_dev=None,
                  stream: int | None = None) -> None:
    """Token ids [T] from bf16 logits [T, V] (``rc_sample_tokens``;
    serve/engine.py:84-140 semantics, uniform draws u_dev [T] f64)."""
    if logits_dev.dim() == 1:
        T, V, ld = 1, int(logits_dev.shape[0]), int(logits_dev.shape[0])
    else:
        T, V = int(logits_dev.shape[0]), int(logits_dev.shape[1])
        ld = int(logits_dev.stride(0))
    check(ctx.lib.rc_sample_tokens(
        ctx.handle, ctypes.c_void_p(_ptr(logits_dev)), ld, T, V, int(top_k), float(top_p), float(temperature),
        float(presence_penalty), ctypes.c_void_p(_ptr(seen_dev)), ctypes.c_void_p(_ptr(seen_off_dev)),
        ctypes.c_void_p(_ptr(u_dev)), ctypes.c_void_p(_ptr(out_dev)),
        ctypes.c_void_p(_stream_for(stream, logits_dev, out_dev))), "rc_sample_tokens")


def add_bf16(ctx: "Context", a_dev, b_dev, out_dev, stream: int | None = None) -> None:
    """out = RTNE(f32(a) + f32(b)) elementwise (bf16 bit tensors of equal size)."""
    n = int(a_dev.numel())
    if int(b_dev.numel()) != n or int(out_dev.numel()) != n:
        raise ValueError("add_bf16: tensors must have the same number of elements")
    check(ctx.lib.rc_add_bf16(ctx.handle, ctypes.c_void_p(_ptr(a_dev)), ctypes.c_void_p(_ptr(b_dev)),
                              ctypes.c_void_p(_ptr(out_dev)), n, ctypes.c_void_p(_stream_for(stream, a_dev, out_dev))),
          "rc_add_bf16")


def add_rms_bf16(ctx: "Context", a_dev, b_dev, out_dev, eps: float = 1e-6, stream: int | None = None) -> None:
    """out = RTNE((a + b) / rms(a + b)) per row of [rows, n] bf16 bit tensors."""
    if a_dev.shape != b_dev.shape or a_dev.shape != out_dev.shape:
        raise ValueError("add_rms_bf16: tensors must have the same shape")
    rows, n = (1, int(a_dev.shape[0])) if a_dev.dim() == 1 else (int(a_dev.shape[0]), int(a_dev.shape[1]))
    check(ctx.lib.rc_add_rms_bf16(ctx.handle, ctypes.c_void_p(_ptr(a_dev)), ctypes.c_void_p(_ptr(b_dev)),
                                  ctypes.c_void_p(_ptr(out_dev)), rows, n, float(eps),
                                  ctypes.c_void_p(_stream_for(stream, a_dev, out_dev))), "rc_add_rms_bf16")


class Q4nxWeight:
    """A q4nx matrix resident in HBM in the GEMV tile layout."""
    _UPLOAD = "rc_upload_q4nx"
    _BITS = 5

    def __init__(self, ctx: Context, packed, n: int, k: int, gate_up: bool = False):
        self.ctx = ctx
        flags = _lib.RC_UPLOAD_GATE_UP if gate_up else 0
        if isinstance(packed, (bytes, bytearray, memoryview, np.ndarray)):
            buf = np.frombuffer(packed, dtype=np.uint8) if not isinstance(packed, np.ndarray) else \
                np.ascontiguousarray(packed, dtype=np.uint8)
            src, nbytes = buf.ctypes.data, buf.nbytes
            keep = buf
        else:  # device tensor: the upload runs on the context stream, so let its producer finish
            flags |= _lib.RC_UPLOAD_SRC_DEVICE
            src, nbytes = _ptr(packed), int(packed.numel() * packed.element_size())
            keep = packed
            if getattr(packed, "is_cuda", False):
                import torch
                torch.cuda.current_stream(packed.device).synchronize()
        h = ctypes.c_void_p()
        check(getattr(ctx.lib, self._UPLOAD)(ctx.handle, ctypes.c_void_p(src), nbytes, int(n), int(k), flags,
                                             ctypes.byref(h)), self._UPLOAD)
        del keep
        self.handle = h
        self.n, self.k, self.gate_up = int(n), int(k), bool(gate_up)
        self.device_bytes = n * k * self._BITS // 8
        ctx._adopt(self)

    def set_bias(self, bias: np.ndarray) -> int:
        """Attach an f32 [n] bias; returns its device address."""
        b = np.ascontiguousarray(bias, dtype=np.float32)
        if b.shape != (self.n,):
            raise ValueError(f"bias must be [{self.n}] float32")
        check(self.ctx.lib.rc_weight_set_bias(self.handle, ctypes.c_void_p(b.ctypes.data)), "rc_weight_set_bias")
        p = ctypes.c_void_p()
        check(self.ctx.lib.rc_weight_bias(self.handle, ctypes.byref(p)))
        return p.value or 0

    def free(self) -> None:
        if self.handle and self.ctx.handle:
            self.ctx.lib.rc_weight_free(self.handle)
        self.handle = None

    release = free

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def dequant_into(self, out_dev, stream: int | None = None) -> None:
        """Write f32 [n, k] weights into a device buffer (bit-exact dequantisation)."""
        check(self.ctx.lib.rc_dequant_q4nx(self.ctx.handle, self.handle, ctypes.c_void_p(_ptr(out_dev)),
                                           ctypes.c_void_p(_stream_for(stream, out_dev))), "rc_dequant_q4nx")

    def gemv_into(self, x_dev, y_dev, tokens: int, x_dtype: int = _lib.RC_DTYPE_BF16, ldx: int | None = None,
                  ldy: int | None = None, row0: int = 0, nrows: int | None = None, bias_dev=None,
                  stream: int | None = None, y_dtype: int | None = None) -> None:
        """Launch ``y = x . W[row0:row0+nrows].T (+bias)`` on device buffers (asynchronous).

        ``y_dtype`` defaults to the activation dtype (the reference contract);
        f32 output with bf16 activations returns the unrounded sums."""
        nrows = self.n - row0 if nrows is None else nrows
        y_dtype = x_dtype if y_dtype is None else y_dtype
        check(self.ctx.lib.rc_gemv(
            self.ctx.handle, self.handle, ctypes.c_void_p(_ptr(x_dev)), int(x_dtype),
            int(self.k if ldx is None else ldx), int(tokens), ctypes.c_void_p(_ptr(y_dev)), int(y_dtype),
            int(nrows if ldy is None else ldy), int(row0), int(nrows), ctypes.c_void_p(_ptr(bias_dev)),
            ctypes.c_void_p(_stream_for(stream, x_dev, y_dev))), "rc_gemv")

    def gemv_noalloc_into(self, x_dev, y_dev, tokens: int, x_dtype: int = _lib.RC_DTYPE_BF16,
                          ldx: int | None = None, ldy: int | None = None, row0: int = 0,
                          nrows: int | None = None, bias_dev=None, stream: int | None = None,
                          y_dtype: int | None = None) -> None:
        """``gemv_into`` through ``rc_gemv_noalloc``: the same result, computed with
        the library's static scratch instead of context-allocated scratch, for
        callers that must not allocate device memory during the call."""
        nrows = self.n - row0 if nrows is None else nrows
        y_dtype = x_dtype if y_dtype is None else y_dtype
        check(self.ctx.lib.rc_gemv_noalloc(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), int(x_dtype), int(self.k if ldx is None else ldx),
            int(tokens), ctypes.c_void_p(_ptr(y_dev)), int(y_dtype), int(nrows if ldy is None else ldy),
            int(row0), int(nrows), ctypes.c_void_p(_ptr(bias_dev)),
            ctypes.c_void_p(_stream_for(stream, x_dev, y_dev))), "rc_gemv_noalloc")

    def gemv_host(self, x: np.ndarray, bias_dev=None) -> np.ndarray:
        """Host-buffer GEMV through ``rc_gemv_host`` (copies in, runs, copies out, waits)."""
        if x.dtype == np.uint16:
            dt, out = _lib.RC_DTYPE_BF16, np.empty((x.shape[0], self.n), np.uint16)
        elif x.dtype == np.float32:
            dt, out = _lib.RC_DTYPE_F32, np.empty((x.shape[0], self.n), np.float32)
        else:
            raise ValueError(f"x must be uint16 (bf16 bits) or float32, got {x.dtype}")
        if x.ndim != 2 or x.shape[1] != self.k:
            raise ValueError(f"x must be [T, {self.k}], got {x.shape}")
        xc = np.ascontiguousarray(x)
        check(self.ctx.lib.rc_gemv_host(self.ctx.handle, self.handle, _np_addr(xc), dt, int(x.shape[0]),
                                        _np_addr(out), _ptr(bias_dev) or None), "rc_gemv_host")
        return out


ACT_CODES = {"swiglu": _lib.RC_ACT_SWIGLU, "situ": _lib.RC_ACT_SITU}
ROUTER_CODES = {"softmax": _lib.RC_ROUTER_SOFTMAX, "sigmoid_bias": _lib.RC_ROUTER_SIGMOID_BIAS}


class Bfp16Weight(Q4nxWeight):
    """A bfp16ebs8 matrix (9-bit block floating point, the reference's
    ``quant/bfp16.py``) resident in HBM in the reference's GEMV packing; used
    through the same ``gemv_into`` / ``gemv_host`` calls (bf16 activations)."""
    _UPLOAD = "rc_upload_bfp16"
    _BITS = 9

    def __init__(self, ctx: Context, packed, n: int, k: int):
        super().__init__(ctx, packed, n, k, gate_up=False)


def _buf(packed):
    """(pointer, nbytes, flags, keepalive) for host bytes/ndarray or a device tensor."""
    if isinstance(packed, (bytes, bytearray, memoryview, np.ndarray)):
        b = np.frombuffer(packed, np.uint8) if not isinstance(packed, np.ndarray) else \
            np.ascontiguousarray(packed, dtype=np.uint8)
        return b.ctypes.data, b.nbytes, 0, b
    if getattr(packed, "is_cuda", False):
        import torch
        torch.cuda.current_stream(packed.device).synchronize()
    return _ptr(packed), int(packed.numel() * packed.element_size()), _lib.RC_UPLOAD_SRC_DEVICE, packed


def _tokens(x, hidden: int) -> int:
    """Token count of an activation tensor [T, hidden] or [hidden]."""
    if x.dim() == 1:
        if x.shape[0] != hidden:
            raise ValueError(f"x must be [hidden={hidden}] or [T, hidden]")
        return 1
    if x.dim() != 2 or x.shape[1] != hidden or not x.is_contiguous():
        raise ValueError(f"x must be a contiguous [T, hidden={hidden}] tensor")
    return int(x.shape[0])


class MoeLayer:
    """One MoE layer on the device: experts (q4nx [gate; up] + down), router.

    ``set_expert`` takes the reference's expert packing (pack_gemv bytes of the
    stacked [gate; up] matrix and of the K-padded down matrix).  For expert
    parallelism, load only the experts a rank owns.
    """

    def __init__(self, ctx: Context, hidden: int, inter: int, n_experts: int, has_shared: bool = True):
        self.ctx = ctx
        h = ctypes.c_void_p()
        check(ctx.lib.rc_moe_create(ctx.handle, int(hidden), int(inter), int(n_experts), int(bool(has_shared)),
                                    ctypes.byref(h)), "rc_moe_create")
        self.handle = h
        self.hidden, self.inter, self.n_experts, self.has_shared = int(hidden), int(inter), int(n_experts), \
            bool(has_shared)
        self.inter_pad = (self.inter + 255) // 256 * 256
        self.loaded: set[int] = set()
        self.down_format = "q4nx"          # of the experts loaded so far (one format per layer)
        ctx._adopt(self)

    def close(self) -> None:
        if self.handle and self.ctx.handle:
            self.ctx.lib.rc_moe_destroy(self.handle)
        self.handle = None

    release = close

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_expert(self, expert: int, gate_up_packed, down_packed, down_format: str = "q4nx") -> None:
        """``down_format="bfp16"``: ``down_packed`` is the bfp16ebs8 GEMV packing
        of the K-padded down matrix (the reference's ``moe_b2`` bundles); every
        expert of a layer must use the same down format."""
        if down_format not in ("q4nx", "bfp16"):
            raise ValueError(f"unknown down format {down_format!r}")
        gp, gn, gf, gk = _buf(gate_up_packed)
        dp, dn, df, dk = _buf(down_packed)
        if gf != df:
            raise ValueError("gate_up and down must both be host or both be device buffers")
        flags = gf | (_lib.RC_UPLOAD_DOWN_BFP16 if down_format == "bfp16" else 0)
        check(self.ctx.lib.rc_moe_set_expert(self.handle, int(expert), ctypes.c_void_p(gp), gn, ctypes.c_void_p(dp),
                                             dn, flags), "rc_moe_set_expert")
        del gk, dk
        self.down_format = down_format
        self.loaded.add(int(expert))

    def set_router(self, router_w_bits: np.ndarray, bias: np.ndarray | None = None) -> None:
        wr = np.ascontiguousarray(router_w_bits, dtype=np.uint16)
        if wr.shape != (self.n_experts, self.hidden):
            raise ValueError(f"router weights must be [{self.n_experts}, {self.hidden}] bf16 bits")
        b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
        if b is not None and b.shape != (self.n_experts,):
            raise ValueError(f"router bias must be [{self.n_experts}] f32")
        check(self.ctx.lib.rc_moe_set_router(self.handle, ctypes.c_void_p(wr.ctypes.data),
                                             ctypes.c_void_p(None if b is None else b.ctypes.data)),
              "rc_moe_set_router")

    def set_fused(self, enable: bool) -> None:
        """Decode through one persistent kernel (default) or separate launches;
        both give the same bytes."""
        check(self.ctx.lib.rc_moe_set_fused(self.handle, int(bool(enable))), "rc_moe_set_fused")

    TRACE_PHASES = ("start", "tokens", "logits", "routed", "selected", "staged", "gate_up", "act_ready", "down",
                    "rows", "end", "keys", "ranked", "act_staged", "down_units", "down_tiles")

    def set_trace(self, stamps_dev, ctas: int = 0) -> None:
        """Phase stamps of the persistent decode kernel (``rc_moe_set_trace``):
        an int64 device buffer of ``ctas`` x 16 global-timer readings, or None
        to switch them off.  Index i of a CTA's row is ``TRACE_PHASES[i]``."""
        check(self.ctx.lib.rc_moe_set_trace(self.handle, ctypes.c_void_p(_ptr(stamps_dev)), int(ctas)),
              "rc_moe_set_trace")

    def set_prefill_kernel(self, kernel: str) -> None:
        """"tcgen05" (default: tensor-core grouped GEMM over 64-token chunks) or
        "gemv" (register-fragment grouped GEMV over 8-token blocks, the decode
        path's bytes)."""
        codes = {"gemv": _lib.RC_PREFILL_GEMV, "tcgen05": _lib.RC_PREFILL_TCGEN05}
        if kernel not in codes:
            raise ValueError(f"unknown prefill kernel {kernel!r}")
        check(self.ctx.lib.rc_moe_set_prefill_kernel(self.handle, codes[kernel]), "rc_moe_set_prefill_kernel")

    def route(self, x_dev, tokens: int, k: int, ids_dev, w_dev, logits_dev=None, router: str = "softmax",
              renormalize: bool = True, scaling: float = 1.0, stream: int | None = None) -> None:
        check(self.ctx.lib.rc_moe_route(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), int(tokens), int(k), ROUTER_CODES[router],
            int(bool(renormalize)), float(scaling), ctypes.c_void_p(_ptr(ids_dev)), ctypes.c_void_p(_ptr(w_dev)),
            ctypes.c_void_p(_ptr(logits_dev)), ctypes.c_void_p(_stream_for(stream, x_dev, ids_dev))), "rc_moe_route")

    def experts(self, x_dev, ids_dev, w_dev, k: int, out_dev, act: str = "situ", gate_beta: float = 4.0,
                value_beta: float = 25.0, with_shared: bool = False, stream: int | None = None) -> None:
        """x [T, hidden] (or [hidden]) bf16, ids / w [T, k] -> out [T, hidden]."""
        check(self.ctx.lib.rc_moe_experts(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), _tokens(x_dev, self.hidden), ctypes.c_void_p(_ptr(ids_dev)),
            ctypes.c_void_p(_ptr(w_dev)), int(k), ACT_CODES[act], float(gate_beta), float(value_beta),
            int(bool(with_shared)), ctypes.c_void_p(_ptr(out_dev)),
            ctypes.c_void_p(_stream_for(stream, x_dev, out_dev))), "rc_moe_experts")

    def experts_host(self, x: np.ndarray, ids: np.ndarray, w: np.ndarray, act: str = "situ", gate_beta: float = 4.0,
                     value_beta: float = 25.0, with_shared: bool = False) -> np.ndarray:
        """Host arrays: x [hidden] or [T, hidden] bf16 bits, ids / w [k] or [T, k]."""
        xh = np.ascontiguousarray(x, dtype=np.uint16)
        ih = np.ascontiguousarray(ids, dtype=np.int32)
        wh = np.ascontiguousarray(w, dtype=np.float32)
        T = 1 if xh.ndim == 1 else xh.shape[0]
        k = ih.shape[-1]
        if xh.shape[-1] != self.hidden or ih.size != T * k or wh.shape != ih.shape:
            raise ValueError("x must be [T, hidden]; ids and weights [T, k]")
        out = np.empty(xh.shape, np.uint16)
        check(self.ctx.lib.rc_moe_experts_host(
            self.handle, ctypes.c_void_p(xh.ctypes.data), T, ctypes.c_void_p(ih.ctypes.data),
            ctypes.c_void_p(wh.ctypes.data), int(k), ACT_CODES[act], float(gate_beta), float(value_beta),
            int(bool(with_shared)), ctypes.c_void_p(out.ctypes.data)), "rc_moe_experts_host")
        return out

    def experts_grouped(self, x_dev, ids_dev, w_dev, k: int, routed_out_dev, shared_gu_dev=None,
                        shared_out_dev=None, act: str = "situ", gate_beta: float = 4.0, value_beta: float = 25.0,
                        stream: int | None = None) -> None:
        """``moe_experts_grouped``: routed sums [T, hidden] and, from the shared
        expert's gate|up rows [T, 2*inter], its down rows [T, hidden]."""
        check(self.ctx.lib.rc_moe_experts_grouped(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), _tokens(x_dev, self.hidden), ctypes.c_void_p(_ptr(ids_dev)),
            ctypes.c_void_p(_ptr(w_dev)), int(k), ctypes.c_void_p(_ptr(shared_gu_dev)), ACT_CODES[act],
            float(gate_beta), float(value_beta), ctypes.c_void_p(_ptr(routed_out_dev)),
            ctypes.c_void_p(_ptr(shared_out_dev)), ctypes.c_void_p(_stream_for(stream, x_dev, routed_out_dev))),
            "rc_moe_experts_grouped")

    def decode(self, x_dev, k: int, out_dev, ids_dev=None, w_dev=None, router: str = "softmax",
               renormalize: bool = True, scaling: float = 1.0, act: str = "swiglu", gate_beta: float = 4.0,
               value_beta: float = 25.0, stream: int | None = None) -> None:
        """x [T, hidden] (or [hidden]) -> out of the same shape; optional ids / w [T, k]."""
        check(self.ctx.lib.rc_moe_decode(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), _tokens(x_dev, self.hidden), int(k), ROUTER_CODES[router],
            int(bool(renormalize)), float(scaling), ACT_CODES[act], float(gate_beta), float(value_beta),
            ctypes.c_void_p(_ptr(out_dev)), ctypes.c_void_p(_ptr(ids_dev)), ctypes.c_void_p(_ptr(w_dev)),
            ctypes.c_void_p(_stream_for(stream, x_dev, out_dev))), "rc_moe_decode")

    def _layer_host(self, fn: str, x: np.ndarray, k: int, routes: bool, stream: int | None, router: str,
                    renormalize: bool, scaling: float, act: str, gate_beta: float, value_beta: float):
        xh = np.ascontiguousarray(x, dtype=np.uint16)
        if xh.shape[-1] != self.hidden or xh.ndim > 2:
            raise ValueError(f"x must be [T, {self.hidden}] bf16 bits, got {xh.shape}")
        T = 1 if xh.ndim == 1 else xh.shape[0]
        out = np.empty(xh.shape, np.uint16)
        ids = np.empty((T, k), np.int32) if routes else None
        w = np.empty((T, k), np.float32) if routes else None
        check(getattr(self.ctx.lib, fn)(
            self.handle, _np_addr(xh), T, int(k), ROUTER_CODES[router], int(bool(renormalize)), float(scaling),
            ACT_CODES[act], float(gate_beta), float(value_beta), _np_addr(out), _np_addr(ids) if routes else None,
            _np_addr(w) if routes else None, _stream_for(stream)), fn)
        return (out, ids, w) if routes else out

    def decode_host(self, x: np.ndarray, k: int, routes: bool = False, stream: int | None = None,
                    router: str = "softmax", renormalize: bool = True, scaling: float = 1.0, act: str = "swiglu",
                    gate_beta: float = 4.0, value_beta: float = 25.0):
        """``decode`` on host arrays through one C call (pinned copies in and
        out, one wait): x [T, hidden] bf16 bits -> out [T, hidden], and with
        ``routes`` also the top-k ids / weights [T, k]."""
        return self._layer_host("rc_moe_decode_host", x, k, routes, stream, router, renormalize, scaling, act,
                                gate_beta, value_beta)

    def prefill_host(self, x: np.ndarray, k: int, routes: bool = False, stream: int | None = None,
                     router: str = "softmax", renormalize: bool = True, scaling: float = 1.0, act: str = "swiglu",
                     gate_beta: float = 4.0, value_beta: float = 25.0):
        """``prefill`` on host arrays, as ``decode_host``."""
        return self._layer_host("rc_moe_prefill_host", x, k, routes, stream, router, renormalize, scaling, act,
                                gate_beta, value_beta)

    def decode_local(self, x_dev, k: int, slot_out_dev, slot_w_dev, experts: tuple[int, int] | None = None,
                     shared_tokens: tuple[int, int] | None = None, router: str = "softmax",
                     renormalize: bool = True, scaling: float = 1.0, act: str = "swiglu", gate_beta: float = 4.0,
                     value_beta: float = 25.0, stream: int | None = None) -> None:
        """Expert-parallel half: slot rows [T, k+1, hidden] of the routed experts
        in ``experts`` = [lo, hi) and of the shared expert for tokens
        ``shared_tokens`` = (t0, count); zeros elsewhere.  Defaults: every
        routed expert, and the shared expert (if any) for every token."""
        T = _tokens(x_dev, self.hidden)
        lo, hi = (0, self.n_experts) if experts is None else (int(experts[0]), int(experts[1]))
        if shared_tokens is None:
            shared_tokens = (0, T) if self.has_shared else (0, 0)
        check(self.ctx.lib.rc_moe_decode_local(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), T, int(k), ROUTER_CODES[router], int(bool(renormalize)),
            float(scaling), ACT_CODES[act], float(gate_beta), float(value_beta), lo, hi, int(shared_tokens[0]),
            int(shared_tokens[1]), ctypes.c_void_p(_ptr(slot_out_dev)), ctypes.c_void_p(_ptr(slot_w_dev)),
            ctypes.c_void_p(_stream_for(stream, x_dev, slot_out_dev))), "rc_moe_decode_local")

    # -- expert parallelism over peer memory ------------------------------
    EP_HANDLE_BYTES = _lib.RC_EP_HANDLE_BYTES

    def ep_init(self, rank: int, world: int, tokens_per_rank: int) -> bytes:
        """Allocates this rank's exchange buffer; returns the blob (IPC handle,
        GPU UUID, geometry) every other rank passes to ``ep_open``."""
        blob = ctypes.create_string_buffer(self.EP_HANDLE_BYTES)
        check(self.ctx.lib.rc_moe_ep_init(self.handle, int(rank), int(world), int(tokens_per_rank),
                                          ctypes.cast(blob, ctypes.c_void_p)), "rc_moe_ep_init")
        return blob.raw

    def ep_open(self, peer: int, blob: bytes) -> None:
        """Maps rank ``peer``'s exchange buffer (a no-op check for this rank's own blob)."""
        if len(blob) != self.EP_HANDLE_BYTES:
            raise ValueError(f"an exchange blob has {self.EP_HANDLE_BYTES} bytes")
        buf = ctypes.create_string_buffer(bytes(blob), self.EP_HANDLE_BYTES)
        check(self.ctx.lib.rc_moe_ep_open(self.handle, int(peer), ctypes.cast(buf, ctypes.c_void_p)),
              "rc_moe_ep_open")

    def ep_decode(self, x_dev, k: int, out_dev, router: str = "softmax", renormalize: bool = True,
                  scaling: float = 1.0, act: str = "swiglu", gate_beta: float = 4.0, value_beta: float = 25.0,
                  stream: int | None = None) -> None:
        """This rank's tokens x [M, hidden] -> out [M, hidden], the exchange with
        the other ranks inside the kernel (every rank calls it together)."""
        check(self.ctx.lib.rc_moe_ep_decode(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), int(k), ROUTER_CODES[router], int(bool(renormalize)),
            float(scaling), ACT_CODES[act], float(gate_beta), float(value_beta), ctypes.c_void_p(_ptr(out_dev)),
            ctypes.c_void_p(_stream_for(stream, x_dev, out_dev))), "rc_moe_ep_decode")

    def ep_decode_host(self, x: np.ndarray, k: int, stream: int | None = None, router: str = "softmax",
                       renormalize: bool = True, scaling: float = 1.0, act: str = "swiglu", gate_beta: float = 4.0,
                       value_beta: float = 25.0) -> np.ndarray:
        """``ep_decode`` on host arrays through one C call: this rank's tokens
        x [M, hidden] bf16 bits -> out [M, hidden]."""
        xh = np.ascontiguousarray(x, dtype=np.uint16)
        if xh.ndim != 2 or xh.shape[1] != self.hidden:
            raise ValueError(f"x must be [M, {self.hidden}] bf16 bits, got {xh.shape}")
        out = np.empty(xh.shape, np.uint16)
        check(self.ctx.lib.rc_moe_ep_decode_host(
            self.handle, _np_addr(xh), int(k), ROUTER_CODES[router], int(bool(renormalize)), float(scaling),
            ACT_CODES[act], float(gate_beta), float(value_beta), _np_addr(out), _stream_for(stream)),
            "rc_moe_ep_decode_host")
        return out

    def prefill(self, x_dev, k: int, out_dev, ids_dev=None, w_dev=None, router: str = "softmax",
                renormalize: bool = True, scaling: float = 1.0, act: str = "swiglu", gate_beta: float = 4.0,
                value_beta: float = 25.0, stream: int | None = None) -> None:
        """The layer for T <= 4096 tokens on the prefill kernel chosen by
        ``set_prefill_kernel``: x [T, hidden] -> out [T, hidden]."""
        check(self.ctx.lib.rc_moe_prefill(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), _tokens(x_dev, self.hidden), int(k), ROUTER_CODES[router],
            int(bool(renormalize)), float(scaling), ACT_CODES[act], float(gate_beta), float(value_beta),
            ctypes.c_void_p(_ptr(out_dev)), ctypes.c_void_p(_ptr(ids_dev)), ctypes.c_void_p(_ptr(w_dev)),
            ctypes.c_void_p(_stream_for(stream, x_dev, out_dev))), "rc_moe_prefill")

    def prefill_experts(self, x_dev, ids_dev, w_dev, k: int, out_dev, act: str = "situ", gate_beta: float = 4.0,
                        value_beta: float = 25.0, with_shared: bool = False, stream: int | None = None) -> None:
        check(self.ctx.lib.rc_moe_prefill_experts(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), _tokens(x_dev, self.hidden), ctypes.c_void_p(_ptr(ids_dev)),
            ctypes.c_void_p(_ptr(w_dev)), int(k), ACT_CODES[act], float(gate_beta), float(value_beta),
            int(bool(with_shared)), ctypes.c_void_p(_ptr(out_dev)),
            ctypes.c_void_p(_stream_for(stream, x_dev, out_dev))), "rc_moe_prefill_experts")

    def prefill_local(self, x_dev, k: int, slot_out_dev, slot_w_dev, experts: tuple[int, int] | None = None,
                      shared_tokens: tuple[int, int] | None = None, router: str = "softmax",
                      renormalize: bool = True, scaling: float = 1.0, act: str = "swiglu", gate_beta: float = 4.0,
                      value_beta: float = 25.0, stream: int | None = None) -> None:
        T = _tokens(x_dev, self.hidden)
        lo, hi = (0, self.n_experts) if experts is None else (int(experts[0]), int(experts[1]))
        if shared_tokens is None:
            shared_tokens = (0, T) if self.has_shared else (0, 0)
        check(self.ctx.lib.rc_moe_prefill_local(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), T, int(k), ROUTER_CODES[router], int(bool(renormalize)),
            float(scaling), ACT_CODES[act], float(gate_beta), float(value_beta), lo, hi, int(shared_tokens[0]),
            int(shared_tokens[1]), ctypes.c_void_p(_ptr(slot_out_dev)), ctypes.c_void_p(_ptr(slot_w_dev)),
            ctypes.c_void_p(_stream_for(stream, x_dev, slot_out_dev))), "rc_moe_prefill_local")

    def prefill_local_routes(self, x_dev, ids_dev, w_dev, k: int, slot_out_dev, slot_w_dev,
                             experts: tuple[int, int] | None = None, shared_tokens: tuple[int, int] | None = None,
                             act: str = "swiglu", gate_beta: float = 4.0, value_beta: float = 25.0,
                             stream: int | None = None, **_router) -> None:
        """``prefill_local`` for given routes ids / w [T, k] (rank order, as
        ``route`` returns them); router options are accepted and ignored."""
        T = _tokens(x_dev, self.hidden)
        lo, hi = (0, self.n_experts) if experts is None else (int(experts[0]), int(experts[1]))
        if shared_tokens is None:
            shared_tokens = (0, T) if self.has_shared else (0, 0)
        check(self.ctx.lib.rc_moe_prefill_local_routes(
            self.handle, ctypes.c_void_p(_ptr(x_dev)), T, ctypes.c_void_p(_ptr(ids_dev)),
            ctypes.c_void_p(_ptr(w_dev)), int(k), ACT_CODES[act], float(gate_beta), float(value_beta), lo, hi,
            int(shared_tokens[0]), int(shared_tokens[1]), ctypes.c_void_p(_ptr(slot_out_dev)),
            ctypes.c_void_p(_ptr(slot_w_dev)), ctypes.c_void_p(_stream_for(stream, x_dev, slot_out_dev))),
            "rc_moe_prefill_local_routes")

    def prefill_combine(self, slot_out_dev, slot_w_dev, k: int, out_dev, tokens: int, with_shared: bool = True,
                        stream: int | None = None) -> None:
        check(self.ctx.lib.rc_moe_prefill_combine(
            self.handle, ctypes.c_void_p(_ptr(slot_out_dev)), ctypes.c_void_p(_ptr(slot_w_dev)), int(tokens),
            int(k), int(bool(with_shared)), ctypes.c_void_p(_ptr(out_dev)),
            ctypes.c_void_p(_stream_for(stream, slot_out_dev, out_dev))), "rc_moe_prefill_combine")

    def combine(self, slot_out_dev, slot_w_dev, k: int, out_dev, tokens: int = 1, with_shared: bool = True,
                stream: int | None = None) -> None:
        """slot rows [T, k+1, hidden] and slot weights [T, k] -> out [T, hidden]."""
        check(self.ctx.lib.rc_moe_combine(
            self.handle, ctypes.c_void_p(_ptr(slot_out_dev)), ctypes.c_void_p(_ptr(slot_w_dev)), int(tokens), int(k),
            int(bool(with_shared)), ctypes.c_void_p(_ptr(out_dev)),
            ctypes.c_void_p(_stream_for(stream, slot_out_dev, out_dev))), "rc_moe_combine")
