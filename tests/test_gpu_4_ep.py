"""Expert parallelism on the GPU: the pair plan of the dispatch step is
checked element by element against the one-device routing, and `world`
ranks' worth of expert shards (run as virtual ranks on one GPU, or as two
NCCL ranks on two GPUs) must reproduce the one-device block and the oracle."""
import os

import numpy as np
import pytest
import torch

import oracle as O
from conftest import ATOL, RTOL, assert_close_bf16, assert_mostly_tight, bf16_np
from gpu_helpers import block_to_oracle
from mlxr_moe import synth
from mlxr_moe.ep import ExpertParallelMoeBlock, loopback_forward
from mlxr_moe.moe import Routing

pytestmark = pytest.mark.gpu

# EP against the one-device block: every element within the north-star bound,
# all but 1e-4 of them within a tighter one (each partial row is rounded to
# bf16 once before the owner adds it up).
TIGHT_ATOL, TIGHT_RTOL, TIGHT_FRAC = 5e-3, 1e-2, 1e-4

_BLOCKS = {}


def block_for(name):
    if name not in _BLOCKS:
        spec = synth.CONFIGS[name]
        _BLOCKS[name] = synth.make_block(spec["cfg"], 0, spec["zipf"])
    return _BLOCKS[name]


def expected_plan(idx, w_u16, world):
    """Host restatement of the dispatch step from one-device routing."""
    T, K = idx.shape
    pairs = {r: [] for r in range(world)}  # r -> [(t, [(local expert, weight bits), ...])]
    first_k = {}
    for t in range(T):
        seen = {}
        for k in range(K):
            e = int(idx[t, k])
            r = e % world
            if r not in seen:
                seen[r] = []
                first_k[(t, r)] = k
                pairs[r].append((t, seen[r]))
            seen[r].append((e // world, int(w_u16[t, k])))
    counts = np.array([[len(pairs[r]), sum(len(s) for _, s in pairs[r])] for r in range(world)], np.int32)
    pair_pos = np.full(T * K, -1, np.int32)
    meta = []
    tok = []
    pos = 0
    for r in range(world):
        for t, slots in pairs[r]:
            pair_pos[t * K + first_k[(t, r)]] = pos
            m = [(le << 16) | wb for le, wb in slots] + [-1] * (K - len(slots))
            meta.append(m)
            tok.append(t)
            pos += 1
    return counts, pair_pos, np.array(meta, np.int64).astype(np.uint32).view(np.int32), np.array(tok)


@pytest.mark.parametrize("name,T,world", [("c1", 32, 8), ("c4", 40, 4), ("c3", 300, 2)])
def test_ep_dispatch_plan_is_exact(name, T, world):
    full = block_for(name)
    cfg = full.cfg
    x = synth.make_input(T, cfg.hidden_size, stream_offset=31)
    r = Routing(T, cfg.num_experts_per_tok, cfg.num_experts, x.device)
    full.forward(x, routing=r)
    blk = ExpertParallelMoeBlock.from_block(full, 0, world)
    ws = blk.workspace(T, 0, 0, x.device)
    plan = blk.dispatch(x, ws)
    torch.cuda.synchronize()
    blk.status()
    idx = r.indices.cpu().numpy().reshape(T, -1)
    wb = bf16_np(r.weights).reshape(T, -1)
    counts, pair_pos, meta, tok = expected_plan(idx, wb, world)
    np.testing.assert_array_equal(plan.send_counts.cpu().numpy(), counts)
    np.testing.assert_array_equal(plan.pair_pos.cpu().numpy()[: T * cfg.num_experts_per_tok], pair_pos)
    P = int(counts[:, 0].sum())
    np.testing.assert_array_equal(plan.meta_send[:P].cpu().numpy(), meta)
    np.testing.assert_array_equal(bf16_np(plan.x_send[:P]), bf16_np(x)[tok])


@pytest.mark.parametrize("name,T,world", [("c1", 32, 2), ("c1", 32, 8), ("c4", 64, 4), ("c3", 512, 2),
                                          ("c5", 96, 8)])
def test_ep_loopback_matches_single_device(name, T, world):
    full = block_for(name)
    blocks = [ExpertParallelMoeBlock.from_block(full, r, world) for r in range(world)]
    xs = [synth.make_input(T, full.cfg.hidden_size, stream_offset=40 + r) for r in range(world)]
    outs = loopback_forward(blocks, xs)
    torch.cuda.synchronize()
    for b in blocks:
        b.status()
    for r in range(world):
        want = full.forward(xs[r])
        torch.cuda.synchronize()
        assert_close_bf16(bf16_np(outs[r]), bf16_np(want), ATOL, RTOL, f"rank {r}")
        assert_mostly_tight(bf16_np(outs[r]), bf16_np(want), TIGHT_ATOL, TIGHT_RTOL, TIGHT_FRAC, f"rank {r} tight")


@pytest.mark.parametrize("name,T,world", [("c3", 256, 4), ("c1", 32, 3)])
def test_ep_loopback_balanced_placement(name, T, world):
    """Experts placed by measured load (uneven counts per rank) give the same
    outputs as one device, and the plan names each expert's rank and local slot."""
    from mlxr_moe.ep import balanced_placement

    full = block_for(name)
    cfg = full.cfg
    xs = [synth.make_input(T, cfg.hidden_size, stream_offset=90 + r) for r in range(world)]
    loads = np.zeros(cfg.num_experts)
    for x in xs:
        idx, _ = full.router(x)
        loads += np.bincount(idx.cpu().numpy().ravel(), minlength=cfg.num_experts)
    place = balanced_placement(loads, world)
    blocks = [ExpertParallelMoeBlock.from_block(full, r, world, place) for r in range(world)]
    per_rank = [sum(loads[e] for e in range(cfg.num_experts) if place[e] == r) for r in range(world)]
    assert max(per_rank) <= loads.sum() / world + loads.max()  # the greedy bound
    outs = loopback_forward(blocks, xs)
    torch.cuda.synchronize()
    for b in blocks:
        b.status()
    for r in range(world):
        want = full.forward(xs[r])
        torch.cuda.synchronize()
        assert_close_bf16(bf16_np(outs[r]), bf16_np(want), ATOL, RTOL, f"rank {r}")
        assert_mostly_tight(bf16_np(outs[r]), bf16_np(want), TIGHT_ATOL, TIGHT_RTOL, TIGHT_FRAC, f"rank {r} tight")


def test_ep_loopback_matches_oracle():
    full = block_for("c1")
    world, T = 4, 32
    blocks = [ExpertParallelMoeBlock.from_block(full, r, world) for r in range(world)]
    xs = [synth.make_input(T, 2048, stream_offset=70 + r) for r in range(world)]
    outs = loopback_forward(blocks, xs)
    torch.cuda.synchronize()
    ocfg, ow = block_to_oracle(full)
    for r in range(world):
        want, _, _ = O.moe_block(ocfg, ow, bf16_np(xs[r]), "fused")
        assert_close_bf16(bf16_np(outs[r]), want, ATOL, RTOL, f"rank {r} vs oracle")
        want_st, _, _ = O.moe_block(ocfg, ow, bf16_np(xs[r]), "staged")
        assert_close_bf16(bf16_np(outs[r]), want_st, ATOL, RTOL, f"rank {r} vs oracle (staged)")


def test_ep_loopback_idle_rank():
    """A rank with no tokens of its own still serves its experts."""
    full = block_for("c4")
    world = 2
    blocks = [ExpertParallelMoeBlock.from_block(full, r, world) for r in range(world)]
    xs = [synth.make_input(48, 2048, stream_offset=80),
          torch.empty((0, 2048), dtype=torch.bfloat16, device="cuda")]
    outs = loopback_forward(blocks, xs)
    torch.cuda.synchronize()
    for b in blocks:
        b.status()
    want = full.forward(xs[0])
    assert outs[1].shape == (0, 2048)
    assert_close_bf16(bf16_np(outs[0]), bf16_np(want), ATOL, RTOL, "rank 0")


def _nccl_worker(rank, world, port, result_path):
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from mlxr_moe.ep import TorchDistExchange

    spec = synth.CONFIGS["c4"]
    full = synth.make_block(spec["cfg"], 0, False, device="cuda")
    blk = ExpertParallelMoeBlock.from_block(full, rank, world)
    ex = TorchDistExchange()
    worst = 0.0
    ok = 1
    for step in range(2):
        x = synth.make_input(48 + 16 * rank, 2048, stream_offset=60 + 4 * rank + step, device="cuda")
        out = blk.forward(x, ex)
        want = full.forward(x)
        torch.cuda.synchronize()
        blk.status()
        err = (out.float() - want.float()).abs()
        worst = max(worst, err.max().item())
        ok &= int(bool((err <= ATOL + RTOL * want.float().abs()).all()))
    t = torch.tensor([ok], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    if rank == 0:
        with open(result_path, "w") as f:
            f.write(f"{int(t.item())} {worst}\n")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_nccl_two_gpus(tmp_path):
    import torch.multiprocessing as mp

    res = tmp_path / "ep.txt"
    mp.spawn(_nccl_worker, args=(2, 29517, str(res)), nprocs=2, join=True)
    ok, err = res.read_text().split()
    assert ok == "1", f"max abs err {err}"


def _p2p_worker(rank, world, port, result_path):
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(rank)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from mlxr_moe.ep import PeerComm, balanced_placement

    worst = 0.0
    ok = 1
    for name, zipf in (("c4", False), ("c3", True)):
        spec = synth.CONFIGS[name]
        cfg = spec["cfg"]
        full = synth.make_block(cfg, 0, spec["zipf"], device="cuda")
        place = None
        if zipf:  # placement from the loads of a calibration batch
            idx, _ = full.router(synth.make_input(64, cfg.hidden_size, stream_offset=7 + rank, device="cuda"))
            loads = torch.bincount(idx.reshape(-1).long(), minlength=cfg.num_experts).to(torch.float64)
            dist.all_reduce(loads)
            place = balanced_placement(loads.cpu().tolist(), world)
        blk = ExpertParallelMoeBlock.from_block(full, rank, world, place)
        comm = PeerComm(rank, world, cap=96, hidden=cfg.hidden_size, k=cfg.num_experts_per_tok)
        # ragged: different token counts per rank and per step, one step with an empty rank
        for step, T in enumerate([48 + 16 * rank, 96 - 40 * rank, 0 if rank == 1 else 33]):
            x = (synth.make_input(T, cfg.hidden_size, stream_offset=100 + 4 * rank + step, device="cuda") if T
                 else torch.empty((0, cfg.hidden_size), dtype=torch.bfloat16, device="cuda"))
            out = blk.forward_p2p(x, comm, device_epoch=zipf)  # c3: the device-resident epoch
            torch.cuda.synchronize()
            blk.status()
            if T:
                want = full.forward(x)
                torch.cuda.synchronize()
                err = (out.float() - want.float()).abs()
                worst = max(worst, err.max().item())
                ok &= int(bool((err <= ATOL + RTOL * want.float().abs()).all()))
        torch.cuda.synchronize()
        dist.barrier()
        comm.close()
        del blk, full
    t = torch.tensor([ok], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    if rank == 0:
        with open(result_path, "w") as f:
            f.write(f"{int(t.item())} {worst}\n")
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_p2p_two_gpus(tmp_path):
    """Exchange inside the kernels over peer memory (CUDA IPC), two GPUs:
    matches the one-device block, ragged and empty batches included; host
    epochs for C4, the device-resident epoch for C3."""
    import torch.multiprocessing as mp

    res = tmp_path / "p2p.txt"
    mp.spawn(_p2p_worker, args=(2, 29519, str(res)), nprocs=2, join=True)
    ok, err = res.read_text().split()
    assert ok == "1", f"max abs err {err}"


@pytest.mark.parametrize("T,world", [(32, 2), (64, 8)])
def test_ep_loopback_gemma4_branch(T, world):
    """The Gemma 4 branch sharded over `world` virtual ranks: the dispatch
    sends the experts' RMS-normed rows, each rank runs its slice of the packed
    gate_up_proj with GeGLU; the outputs match the one-device branch."""
    from mlxr_moe.moe import MoeConfig
    cfg = MoeConfig(1024, 64, 4, 512, bits=4, model_kind=1, rms_norm_eps=1e-6)
    full = synth.make_gemma4_branch(cfg, 0)
    blocks = [ExpertParallelMoeBlock.from_block(full, r, world) for r in range(world)]
    xs = [synth.make_input(T, cfg.hidden_size, stream_offset=60 + r) for r in range(world)]
    outs = loopback_forward(blocks, xs)
    torch.cuda.synchronize()
    for b in blocks:
        b.status()
    for r in range(world):
        want = full.forward(xs[r])
        torch.cuda.synchronize()
        assert_close_bf16(bf16_np(outs[r]), bf16_np(want), ATOL, RTOL, f"rank {r}")
        assert_mostly_tight(bf16_np(outs[r]), bf16_np(want), TIGHT_ATOL, TIGHT_RTOL, TIGHT_FRAC, f"rank {r} tight")


class _OneRankComm:
    """A peer-memory communicator of world 1 (no other process, no IPC): the
    rank's own exchange buffer, created through the C ABI."""

    def __init__(self, cap, hidden, k):
        import ctypes as C

        from mlxr_moe import _lib

        self.comm, self.cap, self.epoch = C.c_void_p(), cap, 0
        handle = (C.c_uint8 * 64)()
        _lib.call("mlxr_cu_ep_comm_create", 1, 0, cap, hidden, k, C.byref(self.comm), handle)

    def close(self):
        from mlxr_moe import _lib

        _lib.call("mlxr_cu_ep_comm_destroy", self.comm)


def test_ep_p2p_one_rank_step_timeout_and_poisoned_flag():
    """The peer-memory step on one GPU with a world-1 communicator: a normal
    step matches the one-device block; an expert step whose epoch no dispatch
    published lets its bounded wait run out and reports MLXR_CU_ERR_TIMEOUT;
    a step whose expert side already failed publishes a poisoned flag, and the
    combine that waits on it reports the failed peer. Every wait here either
    finds its flag set or expires on its own limit."""
    import ctypes as C

    from mlxr_moe import _lib

    full = block_for("c2")
    cfg = full.cfg
    blk = ExpertParallelMoeBlock.from_block(full, 0, 1)
    comm = _OneRankComm(64, cfg.hidden_size, cfg.num_experts_per_tok)
    try:
        x = synth.make_input(40, cfg.hidden_size, stream_offset=77)
        out = blk.forward_p2p(x, comm)
        want = full.forward(x)
        torch.cuda.synchronize()
        blk.status()
        assert_close_bf16(bf16_np(out), bf16_np(want), ATOL, RTOL, "one-rank p2p step")

        ws = blk._ws
        st = torch.cuda.current_stream().cuda_stream
        K, T = cfg.num_experts_per_tok, x.shape[0]
        n_loc = len(blk.experts_here)
        pair_pos = torch.empty(T * K, dtype=torch.int32, device="cuda")

        def experts(epoch):
            _lib.call("mlxr_cu_moe_ep_experts_p2p", C.byref(blk._ccfg), C.byref(blk._cw_loc), n_loc, comm.comm,
                      comm.cap * K, epoch, ws.data_ptr(), ws.numel(), st)

        def dispatch(epoch):
            _lib.call("mlxr_cu_moe_ep_dispatch_p2p", C.byref(blk._ccfg), C.byref(blk._cw_rep), comm.comm,
                      blk.placement.data_ptr(), x.data_ptr(), T, pair_pos.data_ptr(), None, epoch,
                      ws.data_ptr(), ws.numel(), st)

        def combine(epoch):
            _lib.call("mlxr_cu_moe_ep_combine_p2p", C.byref(blk._ccfg), C.byref(blk._cw_rep), comm.comm,
                      x.data_ptr(), T, pair_pos.data_ptr(), None, out.data_ptr(), epoch, ws.data_ptr(),
                      ws.numel(), st)

        # 1. No dispatch published epoch 3: the expert step's wait expires.
        dispatch(2)
        experts(2)
        combine(2)
        blk.status()
        experts(3)
        with pytest.raises(_lib.MlxrError) as e:
            blk.status()
        assert e.value.status == _lib.ERR_TIMEOUT

        # 2. Epoch 4: dispatch is fine, but the status word holds a failure
        # when the expert step publishes, so its flag is poisoned; the combine
        # (status cleared first) finds the poison and reports the failed peer.
        dispatch(4)
        ws[:4].view(torch.int32).fill_(2)
        experts(4)
        ws[:4].view(torch.int32).zero_()
        combine(4)
        with pytest.raises(_lib.MlxrError) as e:
            blk.status()
        assert e.value.status == _lib.ERR_TIMEOUT and "another rank" in e.value.what

        # 3. Epochs outside [1, 2^31) are refused on the host.
        with pytest.raises(_lib.MlxrError):
            experts(0x80000001)
        _lib.LIB.mlxr_cu_clear_error()

        # 4. The next clean step works again.
        dispatch(5)
        experts(5)
        combine(5)
        torch.cuda.synchronize()
        blk.status()
        assert_close_bf16(bf16_np(out), bf16_np(want), ATOL, RTOL, "one-rank p2p step after the failures")
    finally:
        torch.cuda.synchronize()
        comm.close()


def test_ep_p2p_one_rank_device_epoch_and_graph():
    """Steps with the device-resident epoch (epoch 0): steps launched
    directly, then the step captured in a CUDA graph and replayed on new
    inputs (each replay advances the counter in the comm's buffer), all equal
    to the one-device block; a comm that used device epochs refuses host
    epochs."""
    from mlxr_moe import _lib

    full = block_for("c2")
    cfg = full.cfg
    blk = ExpertParallelMoeBlock.from_block(full, 0, 1)
    comm = _OneRankComm(64, cfg.hidden_size, cfg.num_experts_per_tok)
    g = None
    try:
        xs = [synth.make_input(40, cfg.hidden_size, stream_offset=90 + i) for i in range(4)]
        for x in xs[:2]:
            out = blk.forward_p2p(x, comm, device_epoch=True)
            torch.cuda.synchronize()
            blk.status()
            assert_close_bf16(bf16_np(out), bf16_np(full.forward(x)), ATOL, RTOL, "device-epoch step")
        st = torch.cuda.Stream()
        xin, out = xs[0].clone(), torch.empty_like(xs[0])
        with torch.cuda.stream(st):
            blk.forward_p2p(xin, comm, out=out, device_epoch=True)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            blk.forward_p2p(xin, comm, out=out, device_epoch=True)
        for x in xs[2:]:
            with torch.cuda.stream(st):
                xin.copy_(x)
                g.replay()
            torch.cuda.synchronize()
            blk.status()
            assert_close_bf16(bf16_np(out), bf16_np(full.forward(x)), ATOL, RTOL, "replayed device-epoch step")
        with pytest.raises(_lib.MlxrError):
            blk.forward_p2p(xs[0], comm)
    finally:
        del g
        torch.cuda.synchronize()
        comm.close()
