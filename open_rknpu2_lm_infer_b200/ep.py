"""Expert parallelism of the MoE layer across the ranks of a torch.distributed group.

The reference runs every expert of a layer on one device (src/npu/moe.rs); this
module spreads them over G GPUs of one node. Rank g owns the routed experts
[g*P, (g+1)*P), P = E / G, and routes its own tokens (data-parallel rows):

  1. router + top-k on the rank's tokens (the same kernels as one device);
  2. pack: each token is A8-quantised once and one int8 row per kept
     assignment is grouped by destination rank (moe_b200_ep_pack);
  3. counts all-to-all, then rows and (scale, local expert) all-to-all;
  4. the owner of the experts runs the grouped FFN on the rows it received
     (moe_b200_ep_expert_rows), the down GEMM writing in the received order;
  5. the y rows travel back (all-to-all) and the token owner combines them in
     rank order with its routing weights and the residual (moe_b200_ep_combine).

Every row meets the same quantisation, the same GEMM arithmetic and the same
combine order as on one device, so the output is identical to the
single-device layer's bit for bit. The exchange uses NCCL all-to-all
(torch.distributed); the exchange logic itself is written against a small
`ops` interface so that it also runs over gloo ranks on the CPU.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from ._lib import MoeError, check

__all__ = ["ExchangePlan", "ep_forward", "DeviceOps", "DeviceExchange", "ep_forward_device",
           "owner_of"]


def owner_of(expert: np.ndarray, experts_per_rank: int) -> np.ndarray:
    """Rank that owns each (global) expert id."""
    return np.asarray(expert) // experts_per_rank


@dataclass
class ExchangePlan:
    """Host view of one step's exchange: rows sent to / received from each rank."""
    send: list[int]
    recv: list[int]

    @property
    def n_send(self) -> int:
        return sum(self.send)

    @property
    def n_recv(self) -> int:
        return sum(self.recv)


def ep_forward(ops, dist, group, x, residual=None):
    """One expert-parallel layer forward of this rank's tokens `x` [T, H].

    `ops` provides route / pack / expert_rows / combine on the rank's device
    (DeviceOps on a GPU); `dist` is torch.distributed. Returns (out, plan).
    """
    import torch
    ids, routes = ops.route(x)
    send_q, send_scale, send_expert, counts, pos = ops.pack(x, ids, routes)
    recv_counts = torch.empty_like(counts)
    dist.all_to_all_single(recv_counts, counts, group=group)
    plan = ExchangePlan([int(c) for c in counts.tolist()], [int(c) for c in recv_counts.tolist()])
    recv_q = ops.empty_rows(plan.n_recv)
    dist.all_to_all_single(recv_q, send_q[: plan.n_send], plan.recv, plan.send, group=group)
    # scale and local expert travel together as two 32-bit words per row
    meta = torch.stack([send_scale[: plan.n_send].view(torch.int32), send_expert[: plan.n_send]], 1)
    recv_meta = torch.empty((plan.n_recv, 2), dtype=torch.int32, device=meta.device)
    dist.all_to_all_single(recv_meta, meta.contiguous(), plan.recv, plan.send, group=group)
    recv_scale = recv_meta[:, 0].contiguous().view(torch.float32)
    recv_expert = recv_meta[:, 1].contiguous()
    y = ops.expert_rows(recv_q, recv_scale, recv_expert)
    y_back = ops.empty_y(plan.n_send)
    dist.all_to_all_single(y_back, y, plan.send, plan.recv, group=group)
    out = ops.combine(y_back, pos, routes, residual)
    return out, plan


class DeviceOps:
    """The EP steps on one GPU through the C ABI.

    token side: a workspace over all E experts (router, pack, combine) for up
    to `max_rows` tokens; expert side: the rank's bank of P experts with a
    workspace for up to world * max_rows * top received rows."""

    def __init__(self, backend, local_moe, router, world: int, max_rows: int):
        import torch
        self.torch = torch
        self.lib = backend.lib
        self.moe = local_moe
        self.router = router
        self.world = world
        self.hidden = router.hidden
        self.experts = router.experts
        self.top = router.top
        if self.experts % world:
            raise ValueError("the experts must divide evenly over the ranks")
        self.per_rank = self.experts // world
        cfg = backend._config(self.hidden, local_moe.key[1], self.experts, False, self.top, 0)
        cfg.max_rows = max_rows
        raw = self.lib.moe_b200_workspace_create(C.byref(cfg))
        if not raw:
            raise MoeError("cannot allocate the token-side workspace", L.ERR_NOMEM)
        self.ws = raw
        self.row_bytes = int(self.lib.moe_b200_workspace_row_bytes(raw))
        dev = torch.device("cuda", torch.cuda.current_device())
        n = max_rows * self.top
        self.ids = torch.empty((max_rows, self.top), dtype=torch.int32, device=dev)
        self.routes = torch.empty((max_rows, self.top), dtype=torch.float32, device=dev)
        self.send_q = torch.empty((n, self.row_bytes), dtype=torch.int8, device=dev)
        self.send_scale = torch.empty(n, dtype=torch.float32, device=dev)
        self.send_expert = torch.empty(n, dtype=torch.int32, device=dev)
        self.counts = torch.empty(world, dtype=torch.int32, device=dev)
        self.pos = torch.empty(n, dtype=torch.int32, device=dev)
        cap = world * n
        self.recv_q = torch.empty((cap, self.row_bytes), dtype=torch.int8, device=dev)
        self.y = torch.empty((cap, self.hidden), dtype=torch.float32, device=dev)
        self.y_back = torch.empty((n, self.hidden), dtype=torch.float32, device=dev)
        self.out = torch.empty((max_rows, self.hidden), dtype=torch.float32, device=dev)

    def _stream(self):
        return self.torch.cuda.current_stream().cuda_stream

    def route(self, x):
        T = x.shape[0]
        check(self.lib.moe_b200_route_device(self.ws, self.router.raw, T, x.data_ptr(), None,
                                             self.ids.data_ptr(), self.routes.data_ptr(),
                                             self._stream()), "EP router")
        return self.ids[:T], self.routes[:T]

    def pack(self, x, ids, routes):
        T = x.shape[0]
        check(self.lib.moe_b200_ep_pack(self.ws, T, x.data_ptr(), ids.data_ptr(), routes.data_ptr(),
                                        self.per_rank, self.world, self.send_q.data_ptr(),
                                        self.send_scale.data_ptr(), self.send_expert.data_ptr(),
                                        self.counts.data_ptr(), self.pos.data_ptr(),
                                        self._stream()), "EP pack")
        return self.send_q, self.send_scale, self.send_expert, self.counts, self.pos[: T * self.top]

    def empty_rows(self, n):
        return self.recv_q[:n]

    def empty_y(self, n):
        return self.y_back[:n]

    def expert_rows(self, q, scale, expert):
        n = q.shape[0]
        y = self.y[:n]
        check(self.lib.moe_b200_ep_expert_rows(self.moe.workspace, self.moe.weights.raw, n,
                                               q.data_ptr(), scale.data_ptr(), expert.data_ptr(),
                                               y.data_ptr(), self._stream()), "EP expert rows")
        return y

    def combine(self, y_back, pos, routes, residual):
        T = routes.shape[0]
        out = self.out[:T]
        check(self.lib.moe_b200_ep_combine(self.ws, T, y_back.data_ptr(), pos.data_ptr(),
                                           routes.data_ptr(),
                                           None if residual is None else residual.data_ptr(),
                                           out.data_ptr(), self._stream()), "EP combine")
        return out

    def status(self):
        check(self.lib.moe_b200_workspace_status(self.ws), "EP token-side status")
        self.moe.status()

    def close(self):
        if self.ws:
            self.lib.moe_b200_workspace_free(self.ws)
            self.ws = None


class DeviceExchange:
    """The exchange of steps 3-5 done by the GPUs themselves over NVLink peer
    memory (moe_b200_ep_exchange_*): the packed rows are written straight into
    their owners' memory, the owners run their experts, and the expert rows
    come back to the token owners, with the split sizes staying on the device
    (no host synchronisation, so a whole step can be captured in a CUDA
    graph). Setup shares one IPC handle per rank through `dist`
    (all_gather_object); every rank then steps in lockstep."""

    def __init__(self, ops: "DeviceOps", dist, group=None):
        import torch
        self.ops = ops
        self.lib = ops.lib
        rank = dist.get_rank(group) if dist is not None else 0
        world = ops.world
        cap = ops.send_q.shape[0]  # T * top: every packed row of one rank
        raw = self.lib.moe_b200_ep_exchange_create(torch.cuda.current_device(), world, rank, cap,
                                                   ops.row_bytes, ops.hidden)
        if not raw:
            raise MoeError("cannot create the expert-parallel exchange", L.ERR_NOMEM)
        self.raw = raw
        h = (C.c_uint8 * L.EP_HANDLE_BYTES)()
        check(self.lib.moe_b200_ep_exchange_handle(raw, h), "exchange handle")
        mine = bytes(h)
        if world > 1:
            allh = [None] * world
            dist.all_gather_object(allh, mine, group=group)
        else:
            allh = [mine]
        table = (C.c_uint8 * (L.EP_HANDLE_BYTES * world)).from_buffer_copy(b"".join(allh))
        check(self.lib.moe_b200_ep_exchange_connect(raw, table), "exchange connect")
        ptr = self.lib.moe_b200_ep_exchange_y_back(raw)
        self.y_back = torch.as_tensor(_CAI(ptr, (cap, ops.hidden), "<f4"), device="cuda")

    def step(self, send_q, send_scale, send_expert, counts, moe=None):
        """One exchange step; the owners run `moe` (default: the bank of the
        ops this exchange was made with; a layer stack passes each layer's)."""
        moe = self.ops.moe if moe is None else moe
        check(self.lib.moe_b200_ep_exchange_step(
            self.raw, moe.workspace, moe.weights.raw, send_q.data_ptr(),
            send_scale.data_ptr(), send_expert.data_ptr(), counts.data_ptr(), self.ops._stream()),
            "exchange step")
        return self.y_back

    def status(self):
        check(self.lib.moe_b200_ep_exchange_status(self.raw), "exchange status")

    STAGES = ("dispatch_us", "rows_wait_us", "expert_rows_us", "return_us", "return_wait_us")

    def profile(self, enable: bool = True):
        """Record the stage events of the following steps (moe_b200_ep_exchange_profile)."""
        check(self.lib.moe_b200_ep_exchange_profile(self.raw, int(enable)), "exchange profile")

    def profile_read(self) -> dict:
        """Stage times (us) of the last profiled step; waits for it."""
        buf = (C.c_float * 5)()
        check(self.lib.moe_b200_ep_exchange_profile_read(self.raw, buf), "exchange profile read")
        return dict(zip(self.STAGES, (float(v) for v in buf)))

    def probe_timeout(self):
        """Single-rank exchanges: run the row wait on a step nothing completes
        (it gives up after ~2 s; status() then raises the timeout)."""
        check(self.lib.moe_b200_ep_exchange_probe_timeout(self.raw, self.ops._stream()),
              "exchange timeout probe")

    def close(self):
        if self.raw:
            self.lib.moe_b200_ep_exchange_free(self.raw)
            self.raw = None


class _CAI:
    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (ptr, False), "version": 3}


def ep_forward_device(ops: "DeviceOps", ex: DeviceExchange, x, residual=None):
    """ep_forward with the device-initiated exchange: route, pack, exchange
    step, combine; stream-ordered, no host synchronisation."""
    ids, routes = ops.route(x)
    send_q, send_scale, send_expert, counts, pos = ops.pack(x, ids, routes)
    y_back = ex.step(send_q, send_scale, send_expert, counts, ops.moe)
    return ops.combine(y_back, pos, routes, residual)
