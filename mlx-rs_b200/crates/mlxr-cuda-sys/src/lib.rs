//! Raw FFI bindings to libmlxr_moe.so, the B200 (sm_100a) implementation of
//! mlxr's MoE block and its quantised-matmul op family. Hand-written to
//! mirror include/mlxr_moe.h field by field and argument by argument (a CPU
//! test in the library's repository checks the two against each other).
//! Status 0 = success; otherwise mlxr_cu_last_error() holds the message of
//! the calling thread, the contract Guarded::try_from_op already handles
//! (crates/mlxr/src/utils/guard.rs:31-51).
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_int, c_void};

#[repr(C)] #[derive(Clone, Copy)]
pub struct mlxr_cu_moe_config {
    pub hidden_size: i32, pub num_experts: i32, pub num_experts_per_tok: i32,
    pub moe_intermediate_size: i32, pub shared_expert_intermediate_size: i32,
    pub group_size: i32, pub bits: i32, pub shared_bits: i32, pub norm_topk_prob: i32,
    pub shared_gate_bits: i32, // 0 = shared_bits
    pub model_kind: i32,       // 0 Qwen 3.5/3.6 block, 1 Gemma 4 MoE branch
    pub rms_norm_eps: f32,     // model_kind 1
}
#[repr(C)] #[derive(Clone, Copy)]
pub struct mlxr_cu_qlinear { pub weight: *const u32, pub scales: *const c_void, pub biases: *const c_void }
#[repr(C)] #[derive(Clone, Copy)]
pub struct mlxr_cu_moe_weights {
    pub router_weight: *const c_void, pub router_bias: *const f32,
    pub switch_gate: mlxr_cu_qlinear, pub switch_up: mlxr_cu_qlinear, pub switch_down: mlxr_cu_qlinear,
    pub shared_gate: mlxr_cu_qlinear, pub shared_up: mlxr_cu_qlinear, pub shared_down: mlxr_cu_qlinear,
    pub shared_expert_gate: mlxr_cu_qlinear,
    // model_kind 1 (Gemma 4): packed gate_up_proj and the router / experts-input norms
    pub switch_gate_up: mlxr_cu_qlinear,
    pub router_norm: *const c_void, pub expert_scale: *const c_void, pub experts_norm: *const c_void,
}
#[repr(C)]
pub struct mlxr_cu_moe_routing {
    pub indices: *mut i32, pub weights: *mut c_void, pub counts: *mut i32,
    pub offsets: *mut i32, pub sorted_rows: *mut i32, pub inverse: *mut i32,
}

extern "C" {
    pub fn mlxr_cu_last_error() -> *const c_char;
    pub fn mlxr_cu_clear_error();
    pub fn mlxr_cu_abi_version() -> c_int;
    pub fn mlxr_cu_quantize(w: *const c_void, dtype: c_int, rows: i64, cols: i64, group_size: c_int, bits: c_int,
                            mode: *const c_char, wq: *mut u32, scales: *mut c_void, biases: *mut c_void,
                            stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_dequantize(wq: *const u32, scales: *const c_void, biases: *const c_void, sb_dtype: c_int,
                              rows: i64, cols: i64, group_size: c_int, bits: c_int, mode: *const c_char,
                              out: *mut c_void, out_dtype: c_int, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_quantized_matmul(x: *const c_void, x_dtype: c_int, m: i64, k: i64, w: *const u32,
                                    scales: *const c_void, biases: *const c_void, n: i64, transpose: c_int,
                                    group_size: c_int, bits: c_int, mode: *const c_char, out: *mut c_void,
                                    stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_gather_qmm(x: *const c_void, x_dtype: c_int, x_batch: i64, m: i64, k: i64, w: *const u32,
                              scales: *const c_void, biases: *const c_void, w_batch: i64, n: i64,
                              lhs: *const u32, rhs: *const u32, num_indices: i64, transpose: c_int,
                              group_size: c_int, bits: c_int, mode: *const c_char, sorted_indices: c_int,
                              out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_gather_qmm_workspace_size(x_dtype: c_int, x_batch: i64, m: i64, k: i64, w_batch: i64, n: i64,
                                             num_indices: i64, transpose: c_int, group_size: c_int, bits: c_int,
                                             bytes: *mut usize) -> c_int;
    pub fn mlxr_cu_gather_qmm_ws(x: *const c_void, x_dtype: c_int, x_batch: i64, m: i64, k: i64, w: *const u32,
                                 scales: *const c_void, biases: *const c_void, w_batch: i64, n: i64,
                                 lhs: *const u32, rhs: *const u32, num_indices: i64, transpose: c_int,
                                 group_size: c_int, bits: c_int, mode: *const c_char, sorted_indices: c_int,
                                 out: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
                                 stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_quantized_matmul_ws(x: *const c_void, x_dtype: c_int, m: i64, k: i64, w: *const u32,
                                       scales: *const c_void, biases: *const c_void, n: i64, transpose: c_int,
                                       group_size: c_int, bits: c_int, mode: *const c_char, out: *mut c_void,
                                       workspace: *mut c_void, workspace_bytes: usize,
                                       stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_gather_mm(a: *const c_void, b: *const c_void, dtype: c_int, a_batch: i64, m: i64, k: i64,
                             b_batch: i64, n: i64, lhs: *const u32, rhs: *const u32, num_indices: i64,
                             sorted_indices: c_int, out: *mut c_void, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_workspace_size(cfg: *const mlxr_cu_moe_config, num_tokens: i64, bytes: *mut usize) -> c_int;
    pub fn mlxr_cu_moe_block_forward(cfg: *const mlxr_cu_moe_config, weights: *const mlxr_cu_moe_weights,
                                     x: *const c_void, num_tokens: i64, out: *mut c_void,
                                     routing: *const mlxr_cu_moe_routing, workspace: *mut c_void,
                                     workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_block_forward_noalloc(cfg: *const mlxr_cu_moe_config, weights: *const mlxr_cu_moe_weights,
                                             x: *const c_void, num_tokens: i64, out: *mut c_void,
                                             routing: *const mlxr_cu_moe_routing, device_status: *mut c_int,
                                             stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_status(workspace: *const c_void, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_op_status(stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_router(cfg: *const mlxr_cu_moe_config, weights: *const mlxr_cu_moe_weights,
                              x: *const c_void, num_tokens: i64, indices: *mut i32, topk_weights: *mut c_void,
                              logits: *mut c_void, probs: *mut c_void, workspace: *mut c_void,
                              workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_permute(cfg: *const mlxr_cu_moe_config, indices: *const i32, num_tokens: i64,
                               x: *const c_void, counts: *mut i32, offsets: *mut i32, sorted_rows: *mut i32,
                               inverse: *mut i32, x_sorted: *mut c_void, workspace: *mut c_void,
                               workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_experts(cfg: *const mlxr_cu_moe_config, weights: *const mlxr_cu_moe_weights,
                               row_experts: *const i32, num_tokens: i64, x_rows: *const c_void,
                               y_rows: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
                               stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_combine(cfg: *const mlxr_cu_moe_config, weights: *const mlxr_cu_moe_weights,
                               x: *const c_void, num_tokens: i64, y_sorted: *const c_void, inverse: *const i32,
                               topk_weights: *const c_void, out: *mut c_void, workspace: *mut c_void,
                               workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_set_stage_events(events: *const *mut c_void, count: c_int) -> c_int;
    pub fn mlxr_cu_synth_normal_bf16(seed: u64, stream_id: u64, n: i64, stddev: f32, out: *mut c_void,
                                     stream: *mut c_void) -> c_int;
    // expert parallelism (no counterpart in the reference)
    pub fn mlxr_cu_moe_ep_workspace_size(cfg: *const mlxr_cu_moe_config, world: c_int, num_tokens: i64,
                                         max_recv_pairs: i64, max_recv_rows: i64, bytes: *mut usize) -> c_int;
    pub fn mlxr_cu_moe_ep_dispatch(cfg: *const mlxr_cu_moe_config, weights: *const mlxr_cu_moe_weights,
                                   world: c_int, placement: *const i32, x: *const c_void, num_tokens: i64,
                                   send_counts: *mut i32, pair_pos: *mut i32, x_send: *mut c_void,
                                   meta_send: *mut i32, shared_gate: *mut f32, workspace: *mut c_void,
                                   workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_ep_experts(cfg: *const mlxr_cu_moe_config, local_weights: *const mlxr_cu_moe_weights,
                                  num_local_experts: c_int, x_recv: *const c_void, meta_recv: *const i32,
                                  num_pairs: i64, num_rows: i64, partial: *mut c_void, workspace: *mut c_void,
                                  workspace_bytes: usize, stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_ep_combine(cfg: *const mlxr_cu_moe_config, weights: *const mlxr_cu_moe_weights,
                                  x: *const c_void, num_tokens: i64, partial_back: *const c_void, num_pairs: i64,
                                  pair_pos: *const i32, shared_gate: *const f32, out: *mut c_void,
                                  workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> c_int;
    // expert parallelism over peer memory: a communicator per rank, IPC handles
    // (MLXR_CU_IPC_HANDLE_BYTES = 64 each) exchanged by the caller, three steps
    pub fn mlxr_cu_ep_comm_create(world: c_int, rank: c_int, cap: i64, hidden: c_int, k: c_int,
                                  comm: *mut *mut c_void, ipc_handle: *mut c_void) -> c_int;
    pub fn mlxr_cu_ep_comm_connect(comm: *mut c_void, ipc_handles: *const c_void) -> c_int;
    pub fn mlxr_cu_ep_comm_destroy(comm: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_ep_p2p_workspace_size(cfg: *const mlxr_cu_moe_config, comm: *const c_void, num_tokens: i64,
                                             num_local_experts: c_int, expected_rows: i64,
                                             bytes: *mut usize) -> c_int;
    pub fn mlxr_cu_moe_ep_dispatch_p2p(cfg: *const mlxr_cu_moe_config, weights: *const mlxr_cu_moe_weights,
                                       comm: *mut c_void, placement: *const i32, x: *const c_void, num_tokens: i64,
                                       pair_pos: *mut i32, shared_gate: *mut f32, epoch: u32,
                                       workspace: *mut c_void, workspace_bytes: usize,
                                       stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_ep_experts_p2p(cfg: *const mlxr_cu_moe_config, local_weights: *const mlxr_cu_moe_weights,
                                      num_local_experts: c_int, comm: *mut c_void, expected_rows: i64, epoch: u32,
                                      workspace: *mut c_void, workspace_bytes: usize,
                                      stream: *mut c_void) -> c_int;
    pub fn mlxr_cu_moe_ep_combine_p2p(cfg: *const mlxr_cu_moe_config, weights: *const mlxr_cu_moe_weights,
                                      comm: *mut c_void, x: *const c_void, num_tokens: i64, pair_pos: *const i32,
                                      shared_gate: *const f32, out: *mut c_void, epoch: u32,
                                      workspace: *mut c_void, workspace_bytes: usize,
                                      stream: *mut c_void) -> c_int;
}
