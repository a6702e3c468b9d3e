"""Expert-parallel MoE block over several GPUs (one process per GPU).

The reference runs the whole block on one device (Qwen35MoeBlock::forward,
crates/mlxr-lm/src/qwen3_5/text/moe.rs:116-146, has no collective). Here the
experts of a block are spread over `world` ranks: expert e lives on rank
placement[e] (by default e % world; `balanced_placement` spreads measured
expert loads evenly) as that rank's local expert (in increasing expert id);
the router and the shared expert are replicated, so routing is
bit-identical to one device. A step on
each rank:

1. dispatch (`mlxr_cu_moe_ep_dispatch`): route the rank's own tokens and list
   one pair per (token, destination rank) — the token's x row once, plus K
   slots of (local expert, top-k weight) for the experts it has there;
2. exchange the pairs (all-to-all);
3. experts (`mlxr_cu_moe_ep_experts`): run the received pairs through the
   local experts and reduce each pair to one partial row;
4. return the partial rows (the reverse all-to-all);
5. combine (`mlxr_cu_moe_ep_combine`): sum each token's partial rows and add
   the sigmoid-gated shared expert.

`TorchDistExchange` moves the pairs with `torch.distributed` all-to-all
(NCCL over NVLink on GPUs, gloo on CPU for the host-side tests);
`PeerComm` + `ExpertParallelMoeBlock.forward_p2p` do the exchange inside the
kernels over peer memory (CUDA IPC buffers, no collective library and no host
synchronisation per step); `loopback_forward` runs several virtual ranks
inside one process (one GPU).
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .moe import Gemma4MoeBranch, PackedSwitchFfn, QuantizedSwitchLinear, Qwen35MoeBlock, SplitSwitchFfn


def strided_placement(num_experts: int, world: int) -> list[int]:
    """Expert e on rank e % world (the default: neighbouring ids on different ranks)."""
    return [e % world for e in range(num_experts)]


def balanced_placement(loads, world: int) -> list[int]:
    """Longest-processing-time greedy: experts in decreasing load, each to the
    rank with the least load so far (ties: fewer experts, then lower rank).
    `loads` are per-expert row counts measured on a calibration batch; with
    skewed (Zipf) routing this keeps the busiest rank near the mean."""
    loads = [float(v) for v in loads]
    order = sorted(range(len(loads)), key=lambda e: (-loads[e], e))
    tot = [0.0] * world
    cnt = [0] * world
    out = [0] * len(loads)
    for e in order:
        r = min(range(world), key=lambda q: (tot[q], cnt[q], q))
        out[e] = r
        tot[r] += loads[e]
        cnt[r] += 1
    return out


def placement_table(rank_of: list[int]) -> list[int]:
    """(rank << 16) | local index, local indices in increasing expert id."""
    seen: dict[int, int] = {}
    table = []
    for r in rank_of:
        table.append((r << 16) | seen.get(r, 0))
        seen[r] = seen.get(r, 0) + 1
    return table


def _take_experts(q: QuantizedSwitchLinear, experts: list[int]) -> QuantizedSwitchLinear:
    idx = torch.tensor(experts, dtype=torch.long, device=q.weight.device)
    return QuantizedSwitchLinear(q.weight.index_select(0, idx).contiguous(), q.scales.index_select(0, idx).contiguous(),
                                 q.biases.index_select(0, idx).contiguous(), q.group_size, q.bits)


def local_switch(sw, experts: list[int]):
    """The given experts of a switch layer (SplitSwitchFfn, or the Gemma 4
    PackedSwitchFfn), in that order."""
    if isinstance(sw, PackedSwitchFfn):
        return PackedSwitchFfn(_take_experts(sw.gate_up_proj, experts), _take_experts(sw.down_proj, experts))
    return SplitSwitchFfn(*(_take_experts(q, experts) for q in (sw.gate_proj, sw.up_proj, sw.down_proj)))


class DispatchPlan:
    """Outputs of the dispatch step for one rank and step (device tensors)."""

    def __init__(self, T: int, K: int, D: int, world: int, shared: bool, device):
        cap = max(T * min(K, world), 1)
        self.send_counts = torch.zeros((world, 2), dtype=torch.int32, device=device)  # (pairs, filled slots)
        self.pair_pos = torch.empty(max(T * K, 1), dtype=torch.int32, device=device)
        self.x_send = torch.empty((cap, D), dtype=torch.bfloat16, device=device)
        self.meta_send = torch.empty((cap, K), dtype=torch.int32, device=device)
        self.shared_gate = torch.empty(max(T, 1), dtype=torch.float32, device=device) if shared else None
        self.T = T


class ExpertParallelMoeBlock:
    """One rank's share of a Qwen35MoeBlock (or a Gemma4MoeBranch): the router
    and shared expert, or the Gemma 4 router and norms (replicated), and the
    experts that `placement` (rank of each expert; by default e % world) puts
    on this rank."""

    def __init__(self, full: Qwen35MoeBlock, rank: int, world: int, placement: list[int] | None = None):
        cfg = full.cfg
        if world < 1:
            raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, f"world={world} must be >= 1")
        rank_of = list(placement) if placement is not None else strided_placement(cfg.num_experts, world)
        if len(rank_of) != cfg.num_experts or any(r < 0 or r >= world for r in rank_of):
            raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, "placement must give a rank in [0, world) per expert")
        mine = [e for e in range(cfg.num_experts) if rank_of[e] == rank]
        if not mine:
            raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, f"placement leaves rank {rank} without experts")
        self.cfg, self.rank, self.world = cfg, rank, world
        self.rank_of, self.experts_here = rank_of, mine
        self.placement = torch.tensor(placement_table(rank_of), dtype=torch.int32, device=full.gate.device)
        self.gate = full.gate
        self.router_bias = full.router_bias
        self.shared_expert = full.shared_expert
        self.shared_expert_gate = full.shared_expert_gate
        self._ccfg = cfg.to_c()
        z = _lib.QLinear(None, None, None)
        se, seg = self.shared_expert, self.shared_expert_gate
        self._cw_rep = _lib.MoeWeights(
            self.gate.data_ptr(), None if self.router_bias is None else self.router_bias.data_ptr(), z, z, z,
            se.gate_proj.c() if se else z, se.up_proj.c() if se else z, se.down_proj.c() if se else z,
            seg.c() if seg else z)
        if isinstance(full, Gemma4MoeBranch):
            self._norms = (full.router_norm, full.expert_scale, full.experts_norm)  # kept alive with the pointers
            self._cw_rep.router_norm, self._cw_rep.expert_scale, self._cw_rep.experts_norm = (
                t.data_ptr() for t in self._norms)
            self.switch_mlp = local_switch(full.switch_glu, mine)
            sm = self.switch_mlp
            self._cw_loc = _lib.MoeWeights(None, None, z, z, sm.down_proj.c(), z, z, z, z)
            self._cw_loc.switch_gate_up = sm.gate_up_proj.c()
        else:
            self.switch_mlp = local_switch(full.switch_mlp, mine)
            sm = self.switch_mlp
            self._cw_loc = _lib.MoeWeights(None, None, sm.gate_proj.c(), sm.up_proj.c(), sm.down_proj.c(), z, z, z, z)
        self._ws = None

    @classmethod
    def from_block(cls, full: Qwen35MoeBlock, rank: int, world: int,
                   placement: list[int] | None = None) -> "ExpertParallelMoeBlock":
        return cls(full, rank, world, placement)

    def workspace_bytes(self, T: int, max_recv_pairs: int, max_recv_rows: int) -> int:
        n = C.c_size_t(0)
        _lib.call("mlxr_cu_moe_ep_workspace_size", C.byref(self._ccfg), self.world, T, max_recv_pairs,
                  max_recv_rows, C.byref(n))
        return int(n.value)

    def workspace(self, T: int, max_recv_pairs: int, max_recv_rows: int, device) -> torch.Tensor:
        """The step's workspace, grown when a step needs more. A buffer grown
        between the steps of one forward (the received counts are known only
        after the dispatch) starts as a copy of the old one (stream-ordered):
        the experts and combine steps read the status word the dispatch
        cleared."""
        need = self.workspace_bytes(T, max_recv_pairs, max_recv_rows)
        if self._ws is None or self._ws.numel() < need:
            new = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
            if self._ws is not None:
                new[: self._ws.numel()].copy_(self._ws)
            self._ws = new
        return self._ws

    # -- the three device steps --------------------------------------------
    def dispatch(self, x: torch.Tensor, ws: torch.Tensor) -> DispatchPlan:
        T, K = x.shape[0], self.cfg.num_experts_per_tok
        plan = DispatchPlan(T, K, self.cfg.hidden_size, self.world, self.shared_expert is not None, x.device)
        st = torch.cuda.current_stream(x.device).cuda_stream
        _lib.call("mlxr_cu_moe_ep_dispatch", C.byref(self._ccfg), C.byref(self._cw_rep), self.world,
                  self.placement.data_ptr(), x.data_ptr(), T,
                  plan.send_counts.data_ptr(), plan.pair_pos.data_ptr(), plan.x_send.data_ptr(),
                  plan.meta_send.data_ptr(), None if plan.shared_gate is None else plan.shared_gate.data_ptr(),
                  ws.data_ptr(), ws.numel(), st)
        return plan

    def experts(self, x_recv: torch.Tensor, meta_recv: torch.Tensor, num_rows: int, ws: torch.Tensor) -> torch.Tensor:
        P = x_recv.shape[0]
        partial = torch.empty((max(P, 1), self.cfg.hidden_size), dtype=torch.bfloat16, device=x_recv.device)
        st = torch.cuda.current_stream(x_recv.device).cuda_stream
        _lib.call("mlxr_cu_moe_ep_experts", C.byref(self._ccfg), C.byref(self._cw_loc), len(self.experts_here),
                  x_recv.data_ptr(), meta_recv.data_ptr(), P, num_rows, partial.data_ptr(), ws.data_ptr(), ws.numel(),
                  st)
        return partial[:P]

    def combine(self, x: torch.Tensor, partial_back: torch.Tensor, plan: DispatchPlan, ws: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        out = torch.empty_like(x) if out is None else out
        st = torch.cuda.current_stream(x.device).cuda_stream
        P = partial_back.shape[0]
        _lib.call("mlxr_cu_moe_ep_combine", C.byref(self._ccfg), C.byref(self._cw_rep), x.data_ptr(), x.shape[0],
                  partial_back.data_ptr() if P else None, P, plan.pair_pos.data_ptr(),
                  None if plan.shared_gate is None else plan.shared_gate.data_ptr(), out.data_ptr(), ws.data_ptr(),
                  ws.numel(), st)
        return out

    def status(self) -> None:
        """Raises if a device-side check of the last step failed (synchronises)."""
        if self._ws is not None:
            st = torch.cuda.current_stream(self._ws.device).cuda_stream
            _lib.call("mlxr_cu_moe_status", self._ws.data_ptr(), st)

    # -- one step ----------------------------------------------------------
    def forward(self, x: torch.Tensor, exchange: "TorchDistExchange", max_recv_pairs: int | None = None,
                max_recv_rows: int | None = None) -> torch.Tensor:
        """One step on this rank; every rank of the group calls it together.
        With max_recv_* given, the workspace is sized once for those bounds."""
        x = x.reshape(-1, self.cfg.hidden_size).contiguous()
        T = x.shape[0]
        ws = self.workspace(T, max_recv_pairs if max_recv_pairs is not None else 0,
                            max_recv_rows if max_recv_rows is not None else 0, x.device)
        plan = self.dispatch(x, ws)
        recv_counts = exchange.counts(plan.send_counts)
        both = torch.cat([plan.send_counts, recv_counts]).cpu()  # one host sync: the exchange needs the sizes
        send_pairs = both[: self.world, 0].tolist()
        recv_pairs = both[self.world:, 0].tolist()
        recv_rows = int(both[self.world:, 1].sum())
        Ps, Pr = sum(send_pairs), sum(recv_pairs)
        if max_recv_pairs is None or Pr > max_recv_pairs or recv_rows > (max_recv_rows or 0):
            ws = self.workspace(T, Pr, recv_rows, x.device)
        x_recv = exchange.rows(plan.x_send[:Ps], send_pairs, recv_pairs)
        meta_recv = exchange.rows(plan.meta_send[:Ps], send_pairs, recv_pairs)
        partial = self.experts(x_recv, meta_recv, recv_rows, ws)
        back = exchange.rows(partial, recv_pairs, send_pairs)
        return self.combine(x, back, plan, ws)

    def forward_p2p(self, x: torch.Tensor, comm: "PeerComm", expected_rows: int | None = None,
                     out: torch.Tensor | None = None, events=None, device_epoch: bool = False) -> torch.Tensor:
        """One step over peer memory; every rank calls it together (same order of
        steps on every rank, each GPU one rank). events: optional four CUDA
        events recorded on the stream before dispatch, after dispatch, after
        the experts step and after combine (phase timing). device_epoch: the
        step's epoch comes from the comm's device-resident counter (advanced
        by the dispatch), so the step can be captured in a CUDA graph and
        replayed; a comm uses one kind of epoch for its whole life."""
        x = x.reshape(-1, self.cfg.hidden_size).contiguous()
        T, K = x.shape[0], self.cfg.num_experts_per_tok
        if expected_rows is None:
            expected_rows = max(1, comm.cap * K)
        n = C.c_size_t(0)
        _lib.call("mlxr_cu_moe_ep_p2p_workspace_size", C.byref(self._ccfg), comm.comm, T, len(self.experts_here),
                  expected_rows, C.byref(n))
        if self._ws is None or self._ws.numel() < n.value:
            self._ws = torch.empty(max(int(n.value), 256), dtype=torch.uint8, device=x.device)
        ws = self._ws
        mode = "device" if device_epoch else "host"
        if getattr(comm, "epoch_mode", None) not in (None, mode):
            raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT,
                                 f"peer communicator uses {comm.epoch_mode} epochs; a comm keeps one kind")
        comm.epoch_mode = mode
        if device_epoch:
            ep = 0
        else:
            comm.epoch += 1
            if comm.epoch >= 1 << 31:  # the flag's top bit marks a failed step
                raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, "peer communicator ran out of epochs; recreate it")
            ep = comm.epoch
        st = torch.cuda.current_stream(x.device).cuda_stream
        pair_pos = torch.empty(max(T * K, 1), dtype=torch.int32, device=x.device)
        sg = torch.empty(max(T, 1), dtype=torch.float32, device=x.device) if self.shared_expert is not None else None
        out = torch.empty_like(x) if out is None else out
        if events is not None:
            events[0].record()
        _lib.call("mlxr_cu_moe_ep_dispatch_p2p", C.byref(self._ccfg), C.byref(self._cw_rep), comm.comm,
                  self.placement.data_ptr(), x.data_ptr() if T else None, T, pair_pos.data_ptr(),
                  None if sg is None else sg.data_ptr(), ep, ws.data_ptr(), ws.numel(), st)
        if events is not None:
            events[1].record()
        _lib.call("mlxr_cu_moe_ep_experts_p2p", C.byref(self._ccfg), C.byref(self._cw_loc), len(self.experts_here),
                  comm.comm, expected_rows, ep, ws.data_ptr(), ws.numel(), st)
        if events is not None:
            events[2].record()
        _lib.call("mlxr_cu_moe_ep_combine_p2p", C.byref(self._ccfg), C.byref(self._cw_rep), comm.comm,
                  x.data_ptr() if T else None, T, pair_pos.data_ptr(), None if sg is None else sg.data_ptr(),
                  out.data_ptr() if T else None, ep, ws.data_ptr(), ws.numel(), st)
        if events is not None:
            events[3].record()
        return out


class TorchDistExchange:
    """All-to-all of pair rows through torch.distributed (NCCL or gloo).

    Rows travel as raw bytes ([rows, row_bytes] uint8), which every backend
    moves; the split sizes are host lists (the collective needs them there)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group

    def counts(self, send_counts: torch.Tensor) -> torch.Tensor:
        """send_counts [world, c] int32 -> the [world, c] rows the other ranks sent here."""
        recv = torch.empty_like(send_counts)
        w = send_counts.shape[0]
        self.dist.all_to_all_single(recv.view(w, -1).view(torch.uint8), send_counts.contiguous().view(w, -1).view(torch.uint8),
                                    group=self.group)
        return recv

    def rows(self, send: torch.Tensor, send_splits, recv_splits) -> torch.Tensor:
        n = int(sum(recv_splits))
        recv = torch.empty((n,) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        s = send.contiguous().reshape(send.shape[0], -1).view(torch.uint8)
        r = recv.reshape(n, -1).view(torch.uint8)
        self.dist.all_to_all_single(r, s, list(recv_splits), list(send_splits), group=self.group)
        return recv


def loopback_forward(blocks: list[ExpertParallelMoeBlock], xs: list[torch.Tensor]) -> list[torch.Tensor]:
    """One expert-parallel step of `len(blocks)` virtual ranks in this process
    (one device): the exchanges are tensor copies in rank order, exactly the
    layout an all-to-all produces."""
    W = len(blocks)
    K = blocks[0].cfg.num_experts_per_tok
    T_all = sum(x.shape[0] for x in xs)
    wss, plans = [], []
    for b, x in zip(blocks, xs):
        ws = b.workspace(x.shape[0], T_all, T_all * K, x.device)
        wss.append(ws)
        plans.append(b.dispatch(x, ws))
    cnt = [p.send_counts.cpu().tolist() for p in plans]  # cnt[src][dst] = [pairs, rows]
    off = [[sum(cnt[s][d2][0] for d2 in range(d)) for d in range(W)] for s in range(W)]
    partials = []
    for d in range(W):
        xr = torch.cat([plans[s].x_send[off[s][d]: off[s][d] + cnt[s][d][0]] for s in range(W)])
        mr = torch.cat([plans[s].meta_send[off[s][d]: off[s][d] + cnt[s][d][0]] for s in range(W)])
        rows = sum(cnt[s][d][1] for s in range(W))
        partials.append(blocks[d].experts(xr.contiguous(), mr.contiguous(), rows, wss[d]))
    outs = []
    for s in range(W):
        parts = []
        for d in range(W):
            start = sum(cnt[s2][d][0] for s2 in range(s))
            parts.append(partials[d][start: start + cnt[s][d][0]])
        back = torch.cat(parts).contiguous()
        outs.append(blocks[s].combine(xs[s], back, plans[s], wss[s]))
    return outs


class PeerComm:
    """This rank's exchange buffer plus every other rank's, mapped through
    CUDA IPC (`mlxr_cu_ep_comm_create/connect`). The IPC handles travel over
    the `torch.distributed` group (host all-gather, once). `cap` = the most
    tokens any rank feeds a step."""

    def __init__(self, rank: int, world: int, cap: int, hidden: int, k: int, group=None):
        import torch.distributed as dist

        self.rank, self.world, self.cap = rank, world, cap
        self.comm = C.c_void_p()
        handle = (C.c_uint8 * 64)()
        _lib.call("mlxr_cu_ep_comm_create", world, rank, cap, hidden, k, C.byref(self.comm), handle)
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        buf = (C.c_uint8 * (64 * world)).from_buffer_copy(b"".join(handles))
        _lib.call("mlxr_cu_ep_comm_connect", self.comm, buf)
        dist.barrier(group=group)  # every rank has mapped every buffer before the first step
        self.epoch = 0

    def close(self):
        if self.comm:
            _lib.call("mlxr_cu_ep_comm_destroy", self.comm)
            self.comm = C.c_void_p()
