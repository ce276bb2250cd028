"""The ``cuda`` backend: a drop-in for the GEMV / MoE entry points of the
reference's execution backend.

``Backend`` mirrors the hot-path part of the reference ABC
(``host/backend.py:65-204``): the same method names, argument meanings,
return types (bf16 as uint16 bit patterns, f32 in -> f32 out) and exception
classes.  ``CudaBackend`` implements it on the CUDA library; weights are
registered by Hugging Face tensor name, as the reference resolves them
(``npu/backend.py:90-117,3575-3650``), and uploaded once.

The attention / recurrent-state methods of the reference ABC (``rda_update``,
``mla_attend`` and the state get/set) are not part of this path; calling them
raises ``NotImplementedError``.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass

import numpy as np

from . import _lib
from .device import Context, Q4nxWeight


class Backend(ABC):
    """Hot-path subset of the reference ``Backend`` ABC (host/backend.py:65-204)."""

    prefill_shared_precompute: bool = False
    prefill_grouped_moe: bool = False

    def linear_batch(self, name: str, x: np.ndarray) -> np.ndarray:
        """x [T, K] bf16 bits -> [T, N]; byte-identical to stacking ``linear`` per row (host/backend.py:71-74)."""
        return np.stack([self.linear(name, x[t]) for t in range(x.shape[0])])

    @abstractmethod
    def linear(self, name: str, x: np.ndarray) -> np.ndarray:
        """y = x @ W.T (+ bias); ``[..., K]`` input (host/backend.py:76-83)."""

    @abstractmethod
    def moe_experts(self, layer: int, x: np.ndarray, top_ids: np.ndarray, top_weights: np.ndarray,
                    gate_beta: float = 4.0, value_beta: float = 25.0,
                    shared_gu: np.ndarray | None = None) -> np.ndarray:
        """Weighted sum of routed experts for one token (host/backend.py:98-117)."""

    def moe_prestart_shared(self, layer: int, x: np.ndarray) -> None:
        """Overlap hook; results never depend on it (host/backend.py:119-125)."""
        return None

    def moe_abort_prestart_shared(self) -> None:
        return None

    def prefetch_linears(self, items) -> None:
        """Overlap hook; results never depend on it (host/backend.py:131-137)."""
        return None

    def linear_start(self, name: str, x: np.ndarray) -> object:
        """Begin ``linear``; ``linear_finish`` returns exactly ``linear(name, x)`` (host/backend.py:139-155)."""
        return (name, x)

    def linear_finish(self, pending: object) -> np.ndarray:
        name, x = pending
        return self.linear(name, x)

    def linear_abort(self, pending: object) -> None:
        return None


@dataclass
class _Slice:
    bundle: str
    row_start: int
    row_end: int


class CudaBackend(Backend):
    """GEMV / MoE on a B200 through ``libraon_cuda.so``.

    ``register_bundle(bundle, packed, n, k)`` uploads one ``pack_gemv`` matrix;
    ``map_name(name, bundle, row_start, row_end)`` exposes a row slice of it
    under a tensor name (the reference packs several projections into one
    bundle); ``register_q4nx(name, packed, n, k)`` does both for a single
    matrix.  ``orig_k`` lets a matrix whose K was zero-padded to 256 accept the
    unpadded activation (the reference's ``padded_k`` handling).
    """

    def __init__(self, device: int = 0):
        self.ctx = Context(device)
        self._bundles: dict[str, Q4nxWeight] = {}
        self._names: dict[str, _Slice] = {}
        self._orig_k: dict[str, int] = {}
        self._bias: dict[str, int] = {}                   # name -> device address of its bundle's bias
        self._bundle_bias_host: dict[str, np.ndarray] = {}

    # ------------------------------------------------------------ weights --
    def register_bundle(self, bundle: str, packed, n: int, k: int) -> Q4nxWeight:
        if bundle in self._bundles:
            self._bundles[bundle].free()
        w = self.ctx.upload_q4nx(packed, n, k)
        self._bundles[bundle] = w
        return w

    def map_name(self, name: str, bundle: str, row_start: int, row_end: int, orig_k: int | None = None,
                 bias: np.ndarray | None = None) -> None:
        if bundle not in self._bundles:
            raise KeyError(f"Bundle '{bundle}' not registered")
        w = self._bundles[bundle]
        if not 0 <= row_start < row_end <= w.n:
            raise ValueError(f"rows [{row_start}, {row_end}) outside bundle of {w.n} rows")
        self._names[name] = _Slice(bundle, int(row_start), int(row_end))
        if orig_k is not None:
            self._orig_k[name] = int(orig_k)
        if bias is not None:
            b = np.asarray(bias, np.float32)
            if b.shape != (row_end - row_start,):
                raise ValueError(f"bias must be [{row_end - row_start}] f32")
            # One device bias per bundle, holding each named slice's bias at its
            # rows; it is passed only for names that have a bias, so rows
            # without one never see an added +0.0.
            full = self._bundle_bias_host.setdefault(bundle, np.zeros(w.n, np.float32))
            full[row_start:row_end] = b
            self._bias[name] = w.set_bias(full)

    def register_q4nx(self, name: str, packed, n: int, k: int, orig_k: int | None = None,
                      bias: np.ndarray | None = None) -> None:
        self.register_bundle(name, packed, n, k)
        self.map_name(name, name, 0, n, orig_k=orig_k, bias=bias)

    def __contains__(self, name: str) -> bool:
        return name in self._names

    # ------------------------------------------------------------- linear --
    def linear(self, name: str, x: np.ndarray) -> np.ndarray:
        sl = self._names.get(name)
        if sl is None:
            raise KeyError(f"Tensor '{name}' not found in loaded weights.")
        w = self._bundles[sl.bundle]
        x = np.asarray(x)
        if x.dtype not in (np.uint16, np.float32):
            raise ValueError(f"x must be uint16 (bf16 bits) or float32, got {x.dtype}")
        k_in = self._orig_k.get(name, w.k)
        if x.shape[-1] != k_in:
            raise ValueError(f"x last dim {x.shape[-1]} != in-features {k_in} of '{name}'")
        lead = x.shape[:-1]
        x2 = x.reshape(-1, k_in)
        if k_in != w.k:
            xp = np.zeros((x2.shape[0], w.k), x2.dtype)
            xp[:, :k_in] = x2
            x2 = xp
        # The bias (if any) is added in f32 before the output rounding, as the
        # reference does (host/backend.py:410-413).
        y = w.gemv_host(np.ascontiguousarray(x2), bias_dev=self._bias.get(name))
        # Row slices inside a bundle: the kernel works on whole 16-row tiles.
        y = y[:, sl.row_start:sl.row_end]
        return np.ascontiguousarray(y).reshape(*lead, sl.row_end - sl.row_start)

    def linear_batch(self, name: str, x: np.ndarray) -> np.ndarray:
        """One device pass over all T rows; byte-identical to per-row ``linear``."""
        if x.ndim != 2:
            raise ValueError("linear_batch expects x [T, K]")
        return self.linear(name, x)

    # ---------------------------------------------------- out of this path --
    def rda_update(self, *a, **k):
        raise NotImplementedError("rda_update is outside the GEMV/MoE path of this backend")

    def mla_attend(self, *a, **k):
        raise NotImplementedError("mla_attend is outside the GEMV/MoE path of this backend")

    def mla_attend_chunk(self, *a, **k):
        raise NotImplementedError("mla_attend_chunk is outside the GEMV/MoE path of this backend")

    def moe_experts(self, layer, x, top_ids, top_weights, gate_beta=4.0, value_beta=25.0, shared_gu=None):
        raise NotImplementedError("register an MoE layer first")

    def reset(self) -> None:
        return None
