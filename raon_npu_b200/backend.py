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
from .device import Context, MoeLayer, Q4nxWeight


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

    def moe_experts_grouped(self, layer: int, x: np.ndarray, top_ids: np.ndarray, top_weights: np.ndarray,
                            shared_gu: np.ndarray, gate_beta: float = 4.0,
                            value_beta: float = 25.0) -> tuple[np.ndarray, np.ndarray]:
        """Routed sums and shared down rows for T tokens (npu/backend.py:4845-4979)."""
        raise NotImplementedError

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


def _bf16_input(x, hidden: int, what: str) -> np.ndarray:
    """bf16 bits of one token row; f32 rows are rounded (RTNE, NaN -> 0x7FC0)."""
    x = np.asarray(x)
    if x.shape != (hidden,):
        raise ValueError(f"{what} must have shape [{hidden}], got {x.shape}")
    if x.dtype == np.uint16:
        return x
    if x.dtype == np.float32:
        u = x.view(np.uint32).astype(np.uint64)
        r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        r[np.isnan(x)] = 0x7FC0
        return r
    raise ValueError(f"{what} must be uint16 (bf16 bits) or float32, got {x.dtype}")


def check_moe_routes(top_ids, top_weights, n_experts: int, k: int, tokens: int | None = None):
    """The reference's route validation (npu/backend.py:4866-4900, 5047-5056):
    integer ids in range and distinct per token, f32 weights of the same shape.
    Returns (ids int32 [T, k], weights f32 [T, k])."""
    ids = np.asarray(top_ids)
    w = np.asarray(top_weights)
    T = ids.shape[0] if ids.ndim == 2 else -1
    if ids.ndim != 2 or not np.issubdtype(ids.dtype, np.integer) or (tokens is not None and T != tokens) \
            or not 1 <= k <= min(16, n_experts) or ids.shape[1] != k:
        raise ValueError(f"top_ids must be an integer ndarray with shape [T, k], k in 1..{min(16, n_experts)}")
    if np.any(ids < 0) or np.any(ids >= n_experts):
        raise ValueError(f"top_ids values must be in 0..{n_experts - 1}")
    srt = np.sort(ids, axis=1)
    if np.any(srt[:, 1:] == srt[:, :-1]):
        raise ValueError(f"each token must route to {k} distinct experts")
    if w.shape != ids.shape or w.dtype != np.float32:
        raise ValueError(f"top_weights must be a float32 ndarray with shape {ids.shape}")
    return ids.astype(np.int32), w


class CudaBackend(Backend):
    """GEMV / MoE on a B200 through ``libraon_cuda.so``.

    MoE layers: ``register_moe_layer`` + ``register_moe_expert`` per expert;
    ``moe_experts`` / ``moe_experts_grouped`` then run on the device.

    ``register_bundle(bundle, packed, n, k)`` uploads one ``pack_gemv`` matrix;
    ``map_name(name, bundle, row_start, row_end)`` exposes a row slice of it
    under a tensor name (the reference packs several projections into one
    bundle); ``register_q4nx(name, packed, n, k)`` does both for a single
    matrix.  ``orig_k`` lets a matrix whose K was zero-padded to 256 accept the
    unpadded activation (the reference's ``padded_k`` handling).
    """

    prefill_grouped_moe = True

    def __init__(self, device: int = 0):
        self.ctx = Context(device)
        self._bundles: dict[str, Q4nxWeight] = {}
        self._names: dict[str, _Slice] = {}
        self._orig_k: dict[str, int] = {}
        self._bias: dict[str, int] = {}                   # name -> device address of its bundle's bias
        self._bundle_bias_host: dict[str, np.ndarray] = {}
        self._moe: dict[int, tuple[MoeLayer, str]] = {}   # layer -> (experts on the device, activation)

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

    def load_bundles(self, weights_dir):
        """Upload every single-matrix bundle (q4nx or bfp16ebs8) of an exporter
        weights directory (``manifest.json`` + ``*.bin``, size and SHA-256
        checked) and expose each of its components under the component's name
        (a bundle without components under its own name), with the unpadded K
        of ``original_shape`` as the activation width.  Returns the
        ``BundleLoader``; its ``load_moe_experts`` feeds a registered MoE layer
        from expert bundles."""
        from .bundles import GEMV_FORMATS, BundleLoader, Component
        loader = BundleLoader(self.ctx, weights_dir)
        for b in loader.bundles.values():
            if b.fmt not in GEMV_FORMATS:
                continue
            w = loader.upload(b.name)
            old = self._bundles.pop(b.name, None)
            if old is not None:
                old.free()
            self._bundles[b.name] = w
            orig_k = b.original_shape[-1] if b.original_shape[-1] != b.cols else None
            for c in b.components or (Component(b.name, 0, b.original_shape[-2]),):
                self.map_name(c.name, b.name, c.row_start, c.row_end, orig_k=orig_k)
        return loader

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

    # ---------------------------------------------------------------- MoE --
    def register_moe_layer(self, layer: int, hidden: int, inter: int, n_experts: int, act: str = "situ",
                           has_shared: bool = False) -> MoeLayer:
        """Create MoE layer ``layer`` (experts registered with ``register_moe_expert``).
        ``act`` is the GLU of the experts: "situ" (the reference model's) or "swiglu"."""
        if act not in ("situ", "swiglu"):
            raise ValueError(f"unknown activation {act!r}")
        old = self._moe.pop(int(layer), None)
        if old is not None:
            old[0].close()
        m = MoeLayer(self.ctx, hidden, inter, n_experts, has_shared=has_shared)
        self._moe[int(layer)] = (m, act)
        return m

    def register_moe_expert(self, layer: int, expert: int, gate_up_packed, down_packed) -> None:
        """Expert ``expert`` of ``layer`` (``n_experts`` = the shared expert): the
        reference's expert packing (kernels/moe/pack.py:136-224), pack_gemv bytes of
        the stacked [gate; up] matrix and of the K-padded down matrix."""
        self._moe_layer(layer)[0].set_expert(int(expert), gate_up_packed, down_packed)

    def _moe_layer(self, layer):
        if not isinstance(layer, (int, np.integer)):
            raise ValueError("layer must be an integer")
        entry = self._moe.get(int(layer))
        if entry is None:
            raise ValueError(f"layer {layer} is not a registered MoE layer")
        return entry

    def moe_experts(self, layer, x, top_ids, top_weights, gate_beta=4.0, value_beta=25.0, shared_gu=None):
        """Routed experts of one token: ascending-ID f32 sum of w_e * down_e, RTNE
        (host/backend.py:466-510).  f32 ``x`` is rounded to bf16 first, as the
        device backend does (npu/backend.py:5059).  ``shared_gu`` is accepted and
        not used: the shared expert stays with the caller (host/raon.py:1308-1327)."""
        m, act = self._moe_layer(layer)
        x_u16 = _bf16_input(x, m.hidden, "x")
        ids, w = check_moe_routes(np.asarray(top_ids)[None], np.asarray(top_weights)[None], m.n_experts,
                                  np.asarray(top_ids).shape[-1] if np.ndim(top_ids) else 0)
        return m.experts_host(x_u16, ids[0], w[0], act=act, gate_beta=gate_beta, value_beta=value_beta)

    def moe_experts_grouped(self, layer, x, top_ids, top_weights, shared_gu, gate_beta=4.0, value_beta=25.0):
        """T tokens at once (npu/backend.py:4845-4979): returns (routed [T, C],
        shared_down [T, C]), shared_down = down(RTNE(act(shared_gu))) of the
        layer's shared expert.  One device call for the whole batch: up to 16
        tokens on the decode kernels, more (up to 4096) with the routed experts
        on the prefill kernels; a token's bytes are the same either way."""
        import torch
        m, act = self._moe_layer(layer)
        if not isinstance(x, np.ndarray) or x.dtype != np.uint16 or x.ndim != 2 or x.shape[1] != m.hidden \
                or not 1 <= x.shape[0] <= 4096:
            raise ValueError(f"x must be a [T, {m.hidden}] uint16 ndarray with 1 <= T <= 4096")
        T = x.shape[0]
        k = np.asarray(top_ids).shape[-1] if np.ndim(top_ids) == 2 else 0
        ids, w = check_moe_routes(top_ids, top_weights, m.n_experts, k, tokens=T)
        if not m.has_shared:
            raise ValueError(f"layer {layer} has no shared expert")
        if not isinstance(shared_gu, np.ndarray) or shared_gu.dtype != np.uint16 \
                or shared_gu.shape != (T, 2 * m.inter):
            raise ValueError(f"shared_gu must be a [T, {2 * m.inter}] uint16 ndarray")
        dev = torch.device("cuda", self.ctx.device)
        xd = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(dev)
        idd = torch.from_numpy(np.ascontiguousarray(ids)).to(dev)
        wd = torch.from_numpy(np.ascontiguousarray(w)).to(dev)
        gd = torch.from_numpy(np.ascontiguousarray(shared_gu).view(np.int16)).to(dev)
        ro = torch.empty((T, m.hidden), dtype=torch.int16, device=dev)
        so = torch.empty((T, m.hidden), dtype=torch.int16, device=dev)
        m.experts_grouped(xd, idd, wd, k, ro, gd, so, act=act, gate_beta=gate_beta, value_beta=value_beta)
        routed = ro.cpu().numpy().view(np.uint16)
        shared = so.cpu().numpy().view(np.uint16)
        self.ctx.sync()
        return routed, shared

    def reset(self) -> None:
        return None

    def close(self) -> None:
        """Release every device resource of this backend."""
        for m, _ in self._moe.values():
            m.close()
        self._moe.clear()
        for w in self._bundles.values():
            w.free()
        self._bundles.clear()
        self.ctx.close()
