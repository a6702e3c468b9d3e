"""Host-side mirror of the reference's MoE module surface.

Class and method names follow the reference so call sites read the same:
  * QuantizedLinear.forward       crates/mlxr/src/layers/quantized.rs:356-371
  * QuantizedSwitchLinear.apply   crates/mlxr-lm/src/nn/switch.rs:148-167
  * SplitSwitchFfn.forward / forward_with_combine
                                  crates/mlxr-lm/src/nn/switch.rs:417-474
  * SwigluMlp.forward             crates/mlxr-lm/src/nn/swiglu_mlp.rs:63-68
  * Qwen35MoeBlock.forward        crates/mlxr-lm/src/qwen3_5/text/moe.rs:116-146
The op-level classes compose the op family (one C-ABI call per reference op);
Qwen35MoeBlock.forward runs the whole block as one fused call
(mlxr_cu_moe_block_forward) on the current CUDA stream.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib, ops


@dataclass
class MoeConfig:
    """Block dimensions (crates/mlxr-lm/src/qwen3_5/text/config.rs:124-152)."""

    hidden_size: int
    num_experts: int
    num_experts_per_tok: int
    moe_intermediate_size: int
    shared_expert_intermediate_size: int = 0
    group_size: int = 64
    bits: int = 4
    shared_bits: int | None = None
    norm_topk_prob: bool = True
    shared_gate_bits: int | None = None  # None: shared_bits
    model_kind: int = 0                  # 0 Qwen 3.5/3.6 block, 1 Gemma 4 MoE branch (Gemma4MoeBranch)
    rms_norm_eps: float = 1e-6           # model_kind 1: eps of the router and experts-input RMS norms

    def to_c(self) -> _lib.MoeConfig:
        return _lib.MoeConfig(
            self.hidden_size, self.num_experts, self.num_experts_per_tok, self.moe_intermediate_size,
            self.shared_expert_intermediate_size, self.group_size, self.bits,
            self.shared_bits if self.shared_bits is not None else self.bits, int(self.norm_topk_prob),
            self.shared_gate_bits or 0, int(self.model_kind), float(self.rms_norm_eps),
        )


class QuantizedLinear:
    """quantized_matmul(x, w, scales, biases, transpose=true, gs, bits)."""

    def __init__(self, weight, scales, biases, group_size=64, bits=4):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.group_size, self.bits = group_size, bits

    @classmethod
    def from_linear(cls, w: torch.Tensor, group_size=64, bits=4):
        return cls(*ops.quantize(w, group_size, bits), group_size=group_size, bits=bits)

    def forward(self, x):
        return ops.quantized_matmul(x, self.weight, self.scales, self.biases, True, self.group_size, self.bits)

    __call__ = forward

    def c(self) -> _lib.QLinear:
        return _lib.QLinear(self.weight.data_ptr(), self.scales.data_ptr(), self.biases.data_ptr())


class QuantizedSwitchLinear(QuantizedLinear):
    """Per-expert packed weights [E, N, K*bits/32] applied with gather_qmm."""

    @classmethod
    def from_switch_linear(cls, w: torch.Tensor, group_size=64, bits=4):
        return cls(*ops.quantize(w, group_size, bits), group_size=group_size, bits=bits)

    def apply(self, x, indices, sorted_indices=False):
        return ops.gather_qmm(x, self.weight, self.scales, self.biases, None, indices, True, self.group_size,
                              self.bits, sorted_indices)


def swiglu(gate, x):
    """silu(gate) * x (crates/mlxr-lm/src/activations.rs:198-200)."""
    g = gate.float()
    return (g * torch.sigmoid(g) * x.float()).to(gate.dtype)


SORT_THRESHOLD = 2048  # crates/mlxr-lm/src/nn/switch.rs:40


class SplitSwitchFfn:
    """gate_proj / up_proj / down_proj switch linears (switch.rs:367-474), op by op."""

    def __init__(self, gate_proj, up_proj, down_proj):
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj

    def forward(self, x, indices):
        """Per-expert outputs [..., K, D] (switch.rs:417-441)."""
        x_exp = x.unsqueeze(-2).unsqueeze(-3)
        do_sort = indices.numel() >= SORT_THRESHOLD
        if do_sort:
            flat = indices.reshape(-1)
            order = torch.argsort(flat, stable=True)
            inv = torch.argsort(order, stable=True)
            x_flat = x_exp.reshape((-1,) + x_exp.shape[-2:])
            k = indices.shape[-1]
            x_in = x_flat[order // k]
            idx_in = flat[order]
        else:
            x_in, idx_in = x_exp, indices
        g = self.gate_proj.apply(x_in, idx_in, do_sort)
        u = self.up_proj.apply(x_in, idx_in, do_sort)
        y = self.down_proj.apply(swiglu(g, u), idx_in, do_sort)
        if do_sort:
            y = y[inv].reshape(indices.shape + y.shape[-2:])
        return y.squeeze(-2)

    def forward_with_combine(self, x, indices, top_k_weights):
        """sum_k w_k * y_k (switch.rs:446-474)."""
        y = self.forward(x, indices)
        return (top_k_weights.unsqueeze(-1).float() * y.float()).to(y.dtype).sum(-2, dtype=torch.float32).to(y.dtype)


class SwigluMlp:
    """down(swiglu(gate(x), up(x))) (crates/mlxr-lm/src/nn/swiglu_mlp.rs:63-68)."""

    def __init__(self, gate_proj, up_proj, down_proj):
        self.gate_proj, self.up_proj, self.down_proj = gate_proj, up_proj, down_proj

    def forward(self, x):
        return self.down_proj(swiglu(self.gate_proj(x), self.up_proj(x)))


class Routing:
    """Optional routing outputs of Qwen35MoeBlock.forward (device tensors)."""

    def __init__(self, T, K, E, device):
        self.indices = torch.empty((T, K), dtype=torch.int32, device=device)
        self.weights = torch.empty((T, K), dtype=torch.bfloat16, device=device)
        self.counts = torch.empty((E,), dtype=torch.int32, device=device)
        self.offsets = torch.empty((E + 1,), dtype=torch.int32, device=device)
        self.sorted_rows = torch.empty((T * K,), dtype=torch.int32, device=device)
        self.inverse = torch.empty((T * K,), dtype=torch.int32, device=device)

    def c(self) -> _lib.MoeRouting:
        return _lib.MoeRouting(self.indices.data_ptr(), self.weights.data_ptr(), self.counts.data_ptr(),
                               self.offsets.data_ptr(), self.sorted_rows.data_ptr(), self.inverse.data_ptr())


class Qwen35MoeBlock:
    """router -> top-k -> routed SwiGLU experts -> combine (+ gated shared expert).

    Parameters follow moe.rs:52-78: `gate` (router, bf16 [E, D]),
    `switch_mlp` (SplitSwitchFfn of QuantizedSwitchLinear), optional
    `shared_expert` (SwigluMlp of QuantizedLinear) and `shared_expert_gate`
    (QuantizedLinear [1, D]). `router_bias` is an optional fp32 [E] logit bias.
    """

    def __init__(self, cfg: MoeConfig, gate: torch.Tensor, switch_mlp: SplitSwitchFfn,
                 shared_expert: SwigluMlp | None = None, shared_expert_gate: QuantizedLinear | None = None,
                 router_bias: torch.Tensor | None = None):
        self.cfg = cfg
        self.gate = gate.contiguous()
        self.switch_mlp = switch_mlp
        self.shared_expert = shared_expert
        self.shared_expert_gate = shared_expert_gate
        self.router_bias = None if router_bias is None else router_bias.float().contiguous()
        self._ccfg = cfg.to_c()
        self._cw = self._weights_c()
        self._ws = {}

    def _weights_c(self) -> _lib.MoeWeights:
        z = _lib.QLinear(None, None, None)
        sm = self.switch_mlp
        se = self.shared_expert
        return _lib.MoeWeights(
            self.gate.data_ptr(), None if self.router_bias is None else self.router_bias.data_ptr(),
            sm.gate_proj.c(), sm.up_proj.c(), sm.down_proj.c(),
            se.gate_proj.c() if se else z, se.up_proj.c() if se else z, se.down_proj.c() if se else z,
            self.shared_expert_gate.c() if self.shared_expert_gate else z,
        )

    def workspace_bytes(self, num_tokens: int) -> int:
        n = C.c_size_t(0)
        _lib.call("mlxr_cu_moe_workspace_size", C.byref(self._ccfg), num_tokens, C.byref(n))
        return int(n.value)

    def workspace(self, num_tokens: int, device) -> torch.Tensor:
        need = self.workspace_bytes(num_tokens)
        key = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
        ws = self._ws.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
            self._ws[key] = ws
        return ws

    def forward(self, x: torch.Tensor, routing: Routing | None = None, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None) -> torch.Tensor:
        if x.dtype != torch.bfloat16 or not x.is_cuda:
            raise _lib.MlxrError(_lib.ERR_INVALID_ARGUMENT, "Qwen35MoeBlock.forward expects a bf16 CUDA tensor")
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).contiguous()
        T = x2.shape[0]
        if out is None:
            out = torch.empty_like(x2)
        ws = workspace if workspace is not None else self.workspace(T, x.device)
        st = torch.cuda.current_stream(x.device).cuda_stream
        _lib.call("mlxr_cu_moe_block_forward", C.byref(self._ccfg), C.byref(self._cw), x2.data_ptr(), T,
                  out.data_ptr(), C.byref(routing.c()) if routing is not None else None, ws.data_ptr(), ws.numel(), st)
        return out.reshape(shape)

    __call__ = forward

    def status(self, workspace: torch.Tensor | None = None) -> None:
        """Raise if the last forward's device-side status is not OK (synchronises)."""
        ws = workspace if workspace is not None else next(iter(self._ws.values()))
        _lib.call("mlxr_cu_moe_status", ws.data_ptr(), torch.cuda.current_stream(ws.device).cuda_stream)

    def router(self, x: torch.Tensor, want_logits: bool = False):
        """(indices [T,K] int32, weights [T,K] bf16[, logits, probs]) under the routing contract."""
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        T, E, K = x2.shape[0], self.cfg.num_experts, self.cfg.num_experts_per_tok
        idx = torch.empty((T, K), dtype=torch.int32, device=x.device)
        w = torch.empty((T, K), dtype=torch.bfloat16, device=x.device)
        lg = torch.empty((T, E), dtype=torch.bfloat16, device=x.device) if want_logits else None
        pr = torch.empty((T, E), dtype=torch.bfloat16, device=x.device) if want_logits else None
        ws = self.workspace(T, x.device)
        st = torch.cuda.current_stream(x.device).cuda_stream
        _lib.call("mlxr_cu_moe_router", C.byref(self._ccfg), C.byref(self._cw), x2.data_ptr(), T, idx.data_ptr(),
                  w.data_ptr(), None if lg is None else lg.data_ptr(), None if pr is None else pr.data_ptr(),
                  ws.data_ptr(), ws.numel(), st)
        return (idx, w, lg, pr) if want_logits else (idx, w)

    def permute(self, indices: torch.Tensor, x: torch.Tensor):
        """(counts, offsets, sorted_rows, inverse, x_sorted) for routing indices [T, K]."""
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        T, E, K = x2.shape[0], self.cfg.num_experts, self.cfg.num_experts_per_tok
        dev = x.device
        counts = torch.empty(E, dtype=torch.int32, device=dev)
        offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        srt = torch.empty(T * K, dtype=torch.int32, device=dev)
        inv = torch.empty(T * K, dtype=torch.int32, device=dev)
        xs = torch.empty((max(T * K, 1), x2.shape[1]), dtype=torch.bfloat16, device=dev)
        ws = self.workspace(T, dev)
        st = torch.cuda.current_stream(dev).cuda_stream
        _lib.call("mlxr_cu_moe_permute", C.byref(self._ccfg), indices.contiguous().data_ptr(), T, x2.data_ptr(),
                  counts.data_ptr(), offsets.data_ptr(), srt.data_ptr(), inv.data_ptr(), xs.data_ptr(), ws.data_ptr(),
                  ws.numel(), st)
        return counts, offsets, srt, inv, xs[: T * K]

    def experts(self, row_experts: torch.Tensor, x_rows: torch.Tensor) -> torch.Tensor:
        """y_rows [T*K, D]: each row through its expert's SwiGLU FFN, un-weighted (switch.rs:417-442)."""
        K, D = self.cfg.num_experts_per_tok, self.cfg.hidden_size
        R = row_experts.numel()
        if R % K:
            raise ValueError(f"experts: {R} rows is not a multiple of num_experts_per_tok={K}")
        T, dev = R // K, x_rows.device
        xr = x_rows.reshape(R, D).contiguous()
        y = torch.empty((max(R, 1), D), dtype=torch.bfloat16, device=dev)
        ws = self.workspace(T, dev)
        st = torch.cuda.current_stream(dev).cuda_stream
        _lib.call("mlxr_cu_moe_experts", C.byref(self._ccfg), C.byref(self._cw),
                  row_experts.to(torch.int32).contiguous().data_ptr(), T, xr.data_ptr(), y.data_ptr(), ws.data_ptr(),
                  ws.numel(), st)
        return y[:R]

    def combine(self, x: torch.Tensor, y_sorted: torch.Tensor, inverse: torch.Tensor,
                topk_weights: torch.Tensor) -> torch.Tensor:
        """out [T, D]: the weighted sum of each token's expert rows plus the gated shared expert."""
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        T, dev = x2.shape[0], x.device
        out = torch.empty_like(x2)
        ws = self.workspace(T, dev)
        st = torch.cuda.current_stream(dev).cuda_stream
        _lib.call("mlxr_cu_moe_combine", C.byref(self._ccfg), C.byref(self._cw), x2.data_ptr(), T,
                  y_sorted.contiguous().data_ptr(), inverse.to(torch.int32).contiguous().data_ptr(),
                  topk_weights.to(torch.bfloat16).contiguous().data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(),
                  st)
        return out.reshape(x.shape)

    def forward_ops(self, x: torch.Tensor) -> torch.Tensor:
        """The reference's op-by-op chain (moe.rs:116-146) through the op family."""
        idx, w = self.router(x)
        routed = self.switch_mlp.forward_with_combine(x.reshape(-1, x.shape[-1]), idx, w)
        if self.shared_expert is not None:
            x2 = x.reshape(-1, x.shape[-1])
            sh = self.shared_expert.forward(x2)
            sg = torch.sigmoid(self.shared_expert_gate(x2).float()).to(sh.dtype)
            routed = (sh.float() * sg.float()).to(sh.dtype).float() + routed.float()
            routed = routed.to(torch.bfloat16)
        return routed.reshape(x.shape)


class PackedSwitchFfn:
    """Gemma 4 routed experts (nn/switch.rs:242-345): one gate_up_proj switch
    linear [E, 2I, D*b/32] (gate rows 0..I-1, up rows I..2I-1 of each expert)
    and down_proj [E, D, I*b/32], with GeGLU (gelu_approx(gate) * up)."""

    def __init__(self, gate_up_proj: QuantizedSwitchLinear, down_proj: QuantizedSwitchLinear):
        self.gate_up_proj, self.down_proj = gate_up_proj, down_proj


class Gemma4MoeBranch(Qwen35MoeBlock):
    """The Gemma 4 MoE branch of a decoder layer (gemma4/text/text.rs:901-916):
    Router::forward(h) (text.rs:622-664: RMS norm with `router_norm` =
    Router.scale * hidden^-0.5, scores = h_normed . proj, top-k, softmax over
    the k times per_expert_scale) and Experts::forward on
    pre_feedforward_layernorm_2(h) (`experts_norm`), returning the weighted sum
    before post_feedforward_layernorm_2. Same entry points as Qwen35MoeBlock;
    cfg.model_kind must be 1 and there is no shared expert."""

    def __init__(self, cfg: MoeConfig, proj: torch.Tensor, router_norm: torch.Tensor, expert_scale: torch.Tensor,
                 experts_norm: torch.Tensor, switch_glu: PackedSwitchFfn):
        if cfg.model_kind != 1 or cfg.shared_expert_intermediate_size:
            raise ValueError("Gemma4MoeBranch needs model_kind=1 and no shared expert")
        self.router_norm = router_norm.to(torch.bfloat16).contiguous()
        self.expert_scale = expert_scale.to(torch.bfloat16).contiguous()
        self.experts_norm = experts_norm.to(torch.bfloat16).contiguous()
        self.switch_glu = switch_glu
        super().__init__(cfg, proj, None)

    def _weights_c(self) -> _lib.MoeWeights:
        z = _lib.QLinear(None, None, None)
        w = _lib.MoeWeights(self.gate.data_ptr(), None, z, z, self.switch_glu.down_proj.c(), z, z, z, z)
        w.switch_gate_up = self.switch_glu.gate_up_proj.c()
        w.router_norm = self.router_norm.data_ptr()
        w.expert_scale = self.expert_scale.data_ptr()
        w.experts_norm = self.experts_norm.data_ptr()
        return w

    def forward_ops(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError("the op-by-op chain is restated for the Qwen block only")
