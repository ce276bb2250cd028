"""Expert-parallel MoE decode over ``torch.distributed`` (NCCL on B200s).

The reference runs the MoE layer of a decode token on one device
(``host/raon.py:1290-1327``: router, routed experts, shared expert, combine).
Here the routed experts of a layer are split over the ranks of a process
group -- rank r holds experts [r*E/N, (r+1)*E/N) plus a replica of the shared
expert (dense weights stay replicated) -- and each rank decodes its own M
tokens:

1. ``all_gather`` the ranks' token rows -> x [N*M, hidden] on every rank;
2. ``decode_local``: every rank routes all N*M tokens (identical router
   weights and inputs give identical routes everywhere), runs its own experts
   for every token that chose them and the shared expert for its own tokens,
   and writes slot rows [N*M, k+1, hidden] -- zeros where another rank owns
   the slot;
3. ``reduce_scatter`` (sum) of the slot rows: rank r receives the rows of its
   own M tokens.  Every row is non-zero on at most one rank and x + 0 = x in
   bf16, so the sum is exact;
4. ``combine`` (ascending expert ID, f32, then the shared expert) of the own
   tokens.

Prefill (``prefill``) has two exchanges.  "gather" (the default) is the
same four steps over the ranks' whole token sets: all-gather, this rank's
experts over all tokens, reduce-scatter of the slot rows, combine -- fixed
sizes, so a CUDA graph can hold it.  "a2a" sends only the routed rows: every
rank routes its own tokens and exchanges the token rows of remote routes with
their experts' owners in an all-to-all, the owners returning the expert rows
the same way.

The result of every token is byte-identical to the single-GPU decode
(``MoeLayer.decode``): each expert's rows come out of whole-tile GEMVs whose
columns do not interact, the exchange is exact and the combine is the same
kernel.  Two collectives per layer, each a few KB per token.

Transport ``"p2p"`` (the default on NCCL groups whose ranks sit on distinct
GPUs) does all four steps in one persistent kernel per rank
(``MoeLayer.ep_decode``): every rank stores its token rows into every rank's
exchange buffer over NVLink, and each expert row straight into the buffer of
the token's owner -- no collective launches, no zero rows, no sum.  The
buffers are CUDA IPC mappings set up once per token count with one
``all_gather`` of the ranks' handles.  ``"nccl"`` keeps the collectives.
"""

from __future__ import annotations

import numpy as np

from .device import CUDA_STREAM_LEGACY


# rc_moe_route runs the prefill router above this many tokens (the decode
# router below it, whose f64 sums run in another order)
_DECODE_ROUTER_MAX_TOKENS = 16


def _bf16(t):
    import torch
    return t.view(torch.bfloat16)


class ExpertParallelMoe:
    """One MoE layer sharded expert-parallel over ``group``.

    ``layer`` is a :class:`raon_npu_b200.device.MoeLayer` (or an object with
    the same ``decode_local`` / ``combine`` interface and ``n_experts``,
    ``hidden``, ``has_shared`` attributes).  Only the experts this rank owns
    (``owns``) need to be loaded into it.

    ``prefill_exchange``: "gather" (default: all-gather of the token rows,
    this rank's experts over all tokens, reduce-scatter of the slot rows;
    fixed sizes, so a prefill can be captured in a CUDA graph) or "a2a"
    (only the routed rows travel, both ways; split sizes read on the host,
    so the calls are eager).  Both give the single-GPU bytes.
    """

    def __init__(self, layer, k: int, group=None, act: str = "swiglu", router: str = "softmax",
                 renormalize: bool = True, scaling: float = 1.0, gate_beta: float = 4.0, value_beta: float = 25.0,
                 transport: str = "auto", prefill_exchange: str = "gather"):
        import torch.distributed as dist
        self.layer = layer
        self.k = int(k)
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        E = layer.n_experts
        if E % self.world:
            raise ValueError(f"{E} experts do not split evenly over {self.world} ranks")
        per = E // self.world
        self.experts = (self.rank * per, (self.rank + 1) * per)
        self.kw = dict(router=router, renormalize=renormalize, scaling=scaling, act=act, gate_beta=gate_beta,
                       value_beta=value_beta)
        self._bufs: dict = {}
        if transport not in ("auto", "p2p", "nccl"):
            raise ValueError(f"unknown transport {transport!r}")
        if prefill_exchange not in ("gather", "a2a"):
            raise ValueError(f"unknown prefill exchange {prefill_exchange!r}")
        self.prefill_exchange = prefill_exchange
        self.transport = transport
        self._ep_M = None               # token count the peer buffers are set up for (p2p)

    def _use_p2p(self, M: int) -> bool:
        """Whether this call goes through the in-kernel peer exchange; sets the
        buffers up (collectively) the first time a token count is seen."""
        import torch
        import torch.distributed as dist
        if self.transport == "nccl" or self.world == 1:
            return False
        if self._ep_M == M:
            return True
        # the peer-memory kernel computes q4nx down matrices only (every rank's
        # layer has the same format, so every rank decides alike)
        q4nx_down = getattr(self.layer, "down_format", "q4nx") == "q4nx"
        if self.transport == "p2p" and not q4nx_down:
            raise RuntimeError("peer-memory expert parallelism needs q4nx down matrices; use transport='nccl'")
        if self.transport == "auto" and (dist.get_backend(self.group) != "nccl" or self.world * M > 16
                                         or not hasattr(self.layer, "ep_init") or not q4nx_down):
            return False
        # the handshake's tensors live where the group's backend moves them
        on_gpu = dist.get_backend(self.group) == "nccl"
        dev = torch.device("cuda", torch.cuda.current_device()) if on_gpu else torch.device("cpu")
        nb = self.layer.EP_HANDLE_BYTES
        mine = torch.zeros(nb, dtype=torch.uint8, device=dev)
        ok, why = 1, ""
        try:
            mine.copy_(torch.frombuffer(bytearray(self.layer.ep_init(self.rank, self.world, M)), dtype=torch.uint8))
        except Exception as e:          # every rank still takes the collective steps below
            ok, why = 0, str(e)
        blobs = torch.empty(self.world * nb, dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(blobs, mine, group=self.group)
        if ok:
            host = blobs.cpu().numpy().tobytes()
            try:
                for r in range(self.world):
                    self.layer.ep_open(r, host[r * nb:(r + 1) * nb])
            except Exception as e:
                ok, why = 0, str(e)
        flag = torch.tensor([ok], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN, group=self.group)
        if int(flag.item()) == 0:
            if self.transport == "p2p":
                raise RuntimeError(f"peer-memory expert parallelism unavailable: {why or 'failed on another rank'}")
            self.transport = "nccl"
            return False
        self._ep_M = M
        return True

    @property
    def active_transport(self) -> str:
        """The exchange decode calls use now: "p2p" once the peer buffers are
        set up, "nccl" otherwise, "none" on one rank."""
        if self.world == 1:
            return "none"
        return "p2p" if self._ep_M is not None else "nccl"

    def owns(self, expert: int) -> bool:
        """Experts this rank loads: its routed range and the shared expert (id E)."""
        lo, hi = self.experts
        return lo <= expert < hi or (self.layer.has_shared and expert == self.layer.n_experts)

    def _buf(self, name, shape, dtype, device):
        import torch
        b = self._bufs.get(name)
        if b is None or tuple(b.shape) != tuple(shape) or b.device != device:
            b = torch.empty(shape, dtype=dtype, device=device)
            self._bufs[name] = b
        return b

    def decode(self, x, out) -> None:
        """x [M, hidden] bf16 bits (int16) of this rank's tokens -> out [M, hidden]."""
        import torch
        import torch.distributed as dist
        M, H = x.shape
        N, k = self.world, self.k
        if N == 1:                      # nothing to exchange: the single-GPU layer
            self.layer.decode(x, k, out, **self.kw)
            return
        if self._use_p2p(M):
            self.layer.ep_decode(x, k, out, **self.kw)
            return
        T = N * M
        dev = x.device
        if N > 1:
            xg = self._buf("xg", (T, H), torch.int16, dev)
            dist.all_gather_into_tensor(_bf16(xg), _bf16(x), group=self.group)
        else:
            xg = x
        slots = self._buf("slots", (T, k + 1, H), torch.int16, dev)
        sw = self._buf("sw", (T, k), torch.float32, dev)
        shared = (self.rank * M, M) if self.layer.has_shared else (0, 0)
        self.layer.decode_local(xg, k, slots, sw, experts=self.experts, shared_tokens=shared, **self.kw)
        if N > 1:
            mine = self._buf("mine", (M, k + 1, H), torch.int16, dev)
            dist.reduce_scatter_tensor(_bf16(mine), _bf16(slots), op=dist.ReduceOp.SUM, group=self.group)
        else:
            mine = slots
        self.layer.combine(mine, sw[self.rank * M:(self.rank + 1) * M], k, out, tokens=M,
                           with_shared=self.layer.has_shared)

    def prefill(self, x, out) -> None:
        """Prefill of this rank's M tokens x [M, hidden] -> out [M, hidden]
        with the exchange ``prefill_exchange`` names."""
        if self.world == 1:
            self.layer.prefill(x, self.k, out, **self.kw)
        elif self.prefill_exchange == "a2a":
            self.prefill_a2a(x, out)
        else:
            self.prefill_gather(x, out)

    def prefill_gather(self, x, out) -> None:
        """All-gather of every rank's token rows (above 16 tokens per rank with
        their routes: each rank routes only its own tokens); this rank's
        experts for every token that chose them and the shared expert for its
        own tokens (``prefill_local`` / ``prefill_local_routes``: slot rows
        [T, k+1, hidden], zeros where another rank owns the slot);
        reduce-scatter (sum) of the slot rows, exact as each row is non-zero
        on one rank only; ``prefill_combine`` of the own tokens.  Sizes are
        fixed, so it can be captured in a CUDA graph."""
        import torch
        import torch.distributed as dist
        M, H = x.shape
        N, k = self.world, self.k
        T = N * M
        dev = x.device
        xg = self._buf("pxg", (T, H), torch.int16, dev)
        slots = self._buf("pslots", (T, k + 1, H), torch.int16, dev)
        sw = self._buf("psw", (T, k), torch.float32, dev)
        shared = (self.rank * M, M) if self.layer.has_shared else (0, 0)
        if M > _DECODE_ROUTER_MAX_TOKENS and hasattr(self.layer, "prefill_local_routes"):
            # each rank routes only its own tokens (the prefill router, so the
            # routes are those a single GPU computes) and the routes travel
            # with the token rows in one all-gather: row = [x | ids | w]
            route_kw = {n: self.kw[n] for n in ("router", "renormalize", "scaling")}
            ids = self._buf("pids", (M, k), torch.int32, dev)
            wts = self._buf("pw", (M, k), torch.float32, dev)
            self.layer.route(x, M, k, ids, wts, **route_kw)
            W = H + 4 * k
            pk = self._buf("ppk", (M, W), torch.int16, dev)
            pk[:, :H].copy_(x)
            pk[:, H:H + 2 * k].view(torch.int32).copy_(ids)
            pk[:, H + 2 * k:].view(torch.float32).copy_(wts)
            pkg = self._buf("ppkg", (T, W), torch.int16, dev)
            dist.all_gather_into_tensor(_bf16(pkg), _bf16(pk), group=self.group)
            xg.copy_(pkg[:, :H])
            idsg = self._buf("pidsg", (T, k), torch.int32, dev)
            wg = self._buf("pwg", (T, k), torch.float32, dev)
            idsg.copy_(pkg[:, H:H + 2 * k].view(torch.int32))
            wg.copy_(pkg[:, H + 2 * k:].view(torch.float32))
            self.layer.prefill_local_routes(xg, idsg, wg, k, slots, sw, experts=self.experts, shared_tokens=shared,
                                            **self.kw)
        else:
            dist.all_gather_into_tensor(_bf16(xg), _bf16(x), group=self.group)
            self.layer.prefill_local(xg, k, slots, sw, experts=self.experts, shared_tokens=shared, **self.kw)
        mine = self._buf("pmine", (M, k + 1, H), torch.int16, dev)
        dist.reduce_scatter_tensor(_bf16(mine), _bf16(slots), op=dist.ReduceOp.SUM, group=self.group)
        self.last_prefill_exchange = {"rows_sent": (N - 1) * M * (k + 1) + (N - 1) * M,
                                      "rows_received": (N - 1) * M * (k + 1) + (N - 1) * M,
                                      "bytes_sent": 2 * H * ((N - 1) * M * (k + 1) + (N - 1) * M)}
        self.layer.prefill_combine(mine, sw[self.rank * M:(self.rank + 1) * M], k, out, tokens=M,
                                   with_shared=self.layer.has_shared)

    def prefill_a2a(self, x, out) -> None:
        """Prefill of this rank's M tokens x [M, hidden] -> out [M, hidden]
        with an all-to-all exchange of only the routed rows:

        1. route the own tokens on the device (``route``);
        2. every (token, route) becomes a job for the expert's owner, and
           every token a job for the shared expert on this rank; the jobs'
           token rows go to their owners grouped by destination
           (``all_to_all_single``, this rank's own jobs included; the split
           sizes travel first);
        3. each rank runs all the jobs it received in one pass of the prefill
           kernels (``prefill_experts`` with k = 1 and weight 1: the expert's
           bf16 output row, unchanged by the sum), so every local expert's
           weights are streamed once, and sends the rows back in the order
           received;
        4. the rows fill the slots [M, k+1, hidden] (ascending expert ID, the
           shared expert last); ``prefill_combine`` of the own tokens.

        Each expert row comes out of the same tile arithmetic as on one GPU
        (a token's row never depends on the other rows of a pass) and the
        combine is the same kernel, so a token's bytes equal the single-GPU
        prefill.  The split sizes are read on the host, so this path is not
        captured in a CUDA graph."""
        import torch
        import torch.distributed as dist
        M, H = x.shape
        N, k = self.world, self.k
        if N == 1:
            self.layer.prefill(x, k, out, **self.kw)
            return
        if x.is_cuda and torch.cuda.is_current_stream_capturing():
            raise RuntimeError("the expert-parallel prefill sizes its exchange on the host; it cannot be captured")
        dev = x.device
        E = self.layer.n_experts
        per = E // N
        kw = self.kw
        has_shared = self.layer.has_shared
        ids = self._buf("pf_ids", (M, k), torch.int32, dev)
        w = self._buf("pf_w", (M, k), torch.float32, dev)
        self.layer.route(x, M, k, ids, w, router=kw["router"], renormalize=kw["renormalize"],
                         scaling=kw["scaling"])
        ids64 = ids.to(torch.int64)
        # ascending-ID slot of every route; the shared expert takes slot k
        pos = (ids64.unsqueeze(2) > ids64.unsqueeze(1)).sum(dim=2)
        slot_w = torch.zeros((M, k), dtype=torch.float32, device=dev)
        slot_w.scatter_(1, pos, w)
        kj = k + 1 if has_shared else k
        job_e = torch.cat([ids64, torch.full((M, 1), E, dtype=torch.int64, device=dev)], 1) if has_shared else ids64
        job_slot = torch.cat([pos, torch.full((M, 1), k, dtype=torch.int64, device=dev)], 1) if has_shared else pos
        job_e, job_slot = job_e.reshape(-1), job_slot.reshape(-1)
        dest = torch.where(job_e == E, torch.full_like(job_e, self.rank), job_e // per)
        order = torch.argsort(dest * (M * kj) + torch.arange(M * kj, device=dev))   # by destination, token-major
        send_counts = torch.bincount(dest, minlength=N).to(torch.int64)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        send = send_counts.tolist()
        recv = recv_counts.tolist()
        tok = order // kj
        send_x = x[tok].contiguous()
        send_e = job_e[order].to(torch.int32).contiguous()
        n_recv = int(sum(recv))
        recv_x = torch.empty((n_recv, H), dtype=x.dtype, device=dev)
        recv_e = torch.empty((n_recv,), dtype=torch.int32, device=dev)
        dist.all_to_all_single(_bf16(recv_x), _bf16(send_x), output_split_sizes=recv, input_split_sizes=send,
                               group=self.group)
        dist.all_to_all_single(recv_e, send_e, output_split_sizes=recv, input_split_sizes=send, group=self.group)
        rows = torch.empty((n_recv, H), dtype=x.dtype, device=dev)
        if n_recv:
            ones = torch.ones((n_recv, 1), dtype=torch.float32, device=dev)
            self.layer.prefill_experts(recv_x, recv_e.reshape(n_recv, 1), ones, 1, rows, act=kw["act"],
                                       gate_beta=kw["gate_beta"], value_beta=kw["value_beta"], with_shared=False)
        back = torch.empty_like(send_x)
        dist.all_to_all_single(_bf16(back), _bf16(rows), output_split_sizes=send, input_split_sizes=recv,
                               group=self.group)
        slots = self._buf("pf_slots", (M, k + 1, H), torch.int16, dev)
        slots[tok, job_slot[order]] = back
        own = send[self.rank]
        self.last_prefill_exchange = {"rows_sent": int(order.numel()) - own, "rows_received": n_recv - recv[self.rank],
                                      "bytes_sent": 2 * H * (int(order.numel()) - own + n_recv - recv[self.rank])}
        self.layer.prefill_combine(slots, slot_w, k, out, tokens=M, with_shared=has_shared)

    def _host_call(self, x: np.ndarray, run, tag: str) -> np.ndarray:
        """x [M, hidden] bf16 bits on the host -> run(x_dev, out_dev) -> out on
        the host: pinned copies in and out around the call, then a wait."""
        import torch
        xs = np.ascontiguousarray(x, dtype=np.uint16)
        M, H = xs.shape
        dev = torch.device("cuda", torch.cuda.current_device())
        pins = []
        for name in ("in", "out"):
            pin = self._buf(f"{tag}_pin_{name}", (M, H), torch.int16, torch.device("cpu"))
            if not pin.is_pinned():
                pin = pin.pin_memory()
                self._bufs[f"{tag}_pin_{name}"] = pin
            pins.append(pin)
        pin_in, pin_out = pins
        pin_in.numpy()[:] = xs.view(np.int16)
        xd = self._buf(f"{tag}_x_dev", (M, H), torch.int16, dev)
        od = self._buf(f"{tag}_out_dev", (M, H), torch.int16, dev)
        xd.copy_(pin_in, non_blocking=True)
        run(xd, od)
        pin_out.copy_(od, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return pin_out.numpy().copy().view(np.uint16)

    @staticmethod
    def _torch_stream() -> int:
        """The current torch stream as the C ABI takes it (the legacy default
        stream as cudaStreamLegacy), so host calls are ordered after the
        device calls made through the tensors' streams."""
        import torch
        h = int(torch.cuda.current_stream().cuda_stream)
        return h if h != 0 else CUDA_STREAM_LEGACY

    def decode_host(self, x: np.ndarray) -> np.ndarray:
        """Host entry point: x [M, hidden] bf16 bits -> out [M, hidden] (copies in
        from pinned memory, decodes, copies out, waits).  One GPU and the
        peer-memory exchange go through one C call each (the copies, the layer
        and a single wait in native code); the NCCL exchange through torch."""
        xs = np.ascontiguousarray(x, dtype=np.uint16)
        if self.world == 1:
            return self.layer.decode_host(xs, self.k, stream=self._torch_stream(), **self.kw)
        if self._use_p2p(xs.shape[0]):
            return self.layer.ep_decode_host(xs, self.k, stream=self._torch_stream(), **self.kw)
        return self._host_call(xs, self.decode, "dec")

    def prefill_host(self, x: np.ndarray) -> np.ndarray:
        """``prefill`` on host buffers, as ``decode_host`` (one C call on one
        GPU; the collective exchanges through torch)."""
        xs = np.ascontiguousarray(x, dtype=np.uint16)
        if self.world == 1:
            return self.layer.prefill_host(xs, self.k, stream=self._torch_stream(), **self.kw)
        return self._host_call(xs, self.prefill, "pf")
