//! Rust binding of the B200 (sm_100a) kernels of DIAL's quantized-linear hot
//! path: the `extern "C"` declarations of every entry point of
//! `include/dial_cuda.h`, its `#[repr(C)]` structs, and a thin safe layer
//! (status codes to `Result`).
//!
//! The reference's host side sits behind candle's `CustomOp1`
//! (`dial-core/src/models/qwen3_vl/worker_w8a16.rs:388-476`) and `TextLinear`
//! (`worker_w8a16.rs:65-121`); a `TextLinear::Cuda*` variant calls these
//! functions with candle's device pointers and CUDA stream, and maps a
//! non-zero status to `candle_core::Error::Msg(last_error())`.
//!
//! All tensor pointers are device pointers unless the C header says
//! otherwise; `dial_stream` is a `cudaStream_t` (null = the legacy stream).
//! No function allocates device memory: outputs and workspaces come from the
//! caller.

#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_int, c_void, CStr};

pub type dial_status = c_int;
pub const DIAL_OK: dial_status = 0;
pub const DIAL_ERR_INVALID_ARG: dial_status = 1;
pub const DIAL_ERR_UNSUPPORTED_DTYPE: dial_status = 2;
pub const DIAL_ERR_MISALIGNED: dial_status = 3;
pub const DIAL_ERR_SHAPE: dial_status = 4;
pub const DIAL_ERR_CUDA: dial_status = 5;
pub const DIAL_ERR_NCCL: dial_status = 6;
pub const DIAL_ERR_TIMEOUT: dial_status = 7;
pub const DIAL_ERR_NO_DEVICE: dial_status = 8;

pub const DIAL_ABI_VERSION: c_int = 1;

pub type dial_dtype = c_int;
pub const DIAL_F32: dial_dtype = 0;
pub const DIAL_F16: dial_dtype = 1;
pub const DIAL_BF16: dial_dtype = 2;

pub type dial_ggml_type = c_int;
pub const DIAL_GGML_Q4_0: dial_ggml_type = 2;
pub const DIAL_GGML_Q8_0: dial_ggml_type = 8;
pub const DIAL_GGML_Q4_K: dial_ggml_type = 12;
pub const DIAL_GGML_Q6_K: dial_ggml_type = 14;

pub type dial_weight_format = i32;
pub const DIAL_WFMT_W8A16: dial_weight_format = 0;
pub const DIAL_WFMT_W8A16_F16S: dial_weight_format = 1;
pub const DIAL_WFMT_Q4_0: dial_weight_format = 2;
pub const DIAL_WFMT_Q8_0: dial_weight_format = 8;

pub type dial_stream = *mut c_void;

pub const DIAL_PLAN_MASTER: c_int = 0;
pub const DIAL_PLAN_WORKER: c_int = 1;
pub const DIAL_PLAN_MAX_DEVICES: usize = 12;

pub const DIAL_STAGE_COMM_ID_BYTES: usize = 128;

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dial_decoder_dims {
    pub hidden: i32,
    pub intermediate: i32,
    pub n_heads: i32,
    pub n_kv_heads: i32,
    pub head_dim: i32,
    pub vocab: i32,
    pub qk_norm: i32,
    pub weight_format: i32,
    pub head_format: i32,
    pub act_dtype: i32,
    pub rms_eps: f32,
    pub max_seq: i64,
    pub n_slots: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dial_linear_ref {
    pub w: *const c_void,
    pub s: *const c_void,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dial_layer_weights {
    pub qkv: dial_linear_ref,
    pub o: dial_linear_ref,
    pub gate_up: dial_linear_ref,
    pub down: dial_linear_ref,
    pub input_norm: *const c_void,
    pub post_norm: *const c_void,
    pub q_norm: *const c_void,
    pub k_norm: *const c_void,
    pub k_cache: *mut c_void,
    pub v_cache: *mut c_void,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dial_layer_metric {
    pub per_layer: *const f64,
    pub uniform: f64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dial_plan_device {
    pub role: c_int,
    pub enabled: c_int,
    pub usable_memory_mb: f64,
    pub fixed_memory_mb: f64,
    pub layer_memory_mb: dial_layer_metric,
    pub prefill_ms: dial_layer_metric,
    pub decode_ms: dial_layer_metric,
    pub has_prefill_p95: c_int,
    pub has_decode_p95: c_int,
    pub prefill_p95_ms: dial_layer_metric,
    pub decode_p95_ms: dial_layer_metric,
    pub prefill_energy_mj: dial_layer_metric,
    pub decode_energy_mj: dial_layer_metric,
    pub rtt_ms: f64,
    pub protocol_ms: f64,
    pub bandwidth_mbps: f64,
    pub rtt_p95_ms: f64,
    pub protocol_p95_ms: f64,
    pub bandwidth_p05_mbps: f64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dial_plan_objective {
    pub prompt_tokens: c_int,
    pub output_tokens: c_int,
    pub dtype_bytes: c_int,
    pub kv_context_tokens: c_int,
    pub ttft_weight: f64,
    pub tpot_weight: f64,
    pub risk_weight: f64,
    pub energy_weight: f64,
    pub remote_device_penalty: f64,
    pub min_devices: c_int,
    pub max_devices: c_int,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct dial_plan_model {
    pub num_layers: c_int,
    pub hidden_size: c_int,
    pub num_attention_heads: c_int,
    pub num_key_value_heads: c_int,
    pub max_seq_len: c_int,
    pub head_memory_mb: f64,
    pub head_prefill_ms: f64,
    pub head_decode_ms: f64,
    pub embed_memory_mb: f64,
    pub embed_prefill_ms: f64,
    pub embed_decode_ms: f64,
    pub link_topology: c_int,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct dial_plan_segment {
    pub device: c_int,
    pub start_layer: c_int,
    pub end_layer: c_int,
    pub memory_mb: f64,
    pub ttft_ms: f64,
    pub tpot_ms: f64,
    pub tail_ttft_ms: f64,
    pub tail_tpot_ms: f64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct dial_plan_result {
    pub n_segments: c_int,
    pub segments: [dial_plan_segment; DIAL_PLAN_MAX_DEVICES],
    pub ttft_ms: f64,
    pub tpot_ms: f64,
    pub tail_ttft_ms: f64,
    pub tail_tpot_ms: f64,
    pub request_energy_mj: f64,
    pub score: f64,
    pub states_considered: i64,
    pub feasible_transitions: i64,
    pub rejected_for_memory: i64,
}

/// Opaque NCCL stage communicator (one pipeline link).
#[repr(C)]
pub struct dial_stage_comm {
    _private: [u8; 0],
}

extern "C" {
    // misc
    pub fn dial_status_string(s: dial_status) -> *const c_char;
    pub fn dial_last_error() -> *const c_char;
    pub fn dial_abi_version() -> c_int;
    pub fn dial_launch_count() -> u64;
    pub fn dial_device_error(clear: c_int) -> dial_status;
    pub fn dial_check_bounded_wait(src: *const c_void, result: *mut i32, stream: dial_stream) -> dial_status;

    // W8A16 (CudaW8A16Linear, worker_w8a16.rs:291-476)
    pub fn dial_w8a16_quantize(w: *const c_void, wdt: dial_dtype, n: i64, k: i64, q: *mut i8,
                               scale: *mut c_void, sdt: dial_dtype, stream: dial_stream) -> dial_status;
    pub fn dial_w8a16_dequantize(q: *const i8, scale: *const c_void, sdt: dial_dtype, n: i64, k: i64,
                                 w: *mut c_void, wdt: dial_dtype, stream: dial_stream) -> dial_status;
    pub fn dial_w8a16_linear_workspace_bytes(n: i64) -> usize;
    pub fn dial_w8a16_linear(x: *const c_void, xdt: dial_dtype, q: *const i8, scale: *const c_void,
                             sdt: dial_dtype, y: *mut c_void, m: i64, k: i64, n: i64,
                             workspace: *mut c_void, workspace_bytes: usize,
                             stream: dial_stream) -> dial_status;

    // GGUF Q4_0 / Q8_0 (load_worker_gguf_linear / forward_worker_gguf, worker_gguf.rs:462-611)
    pub fn dial_gguf_qs_bytes(ty: dial_ggml_type, n: i64, k: i64) -> usize;
    pub fn dial_gguf_d_bytes(n: i64, k: i64) -> usize;
    pub fn dial_gguf_repack(blocks: *const c_void, ty: dial_ggml_type, n: i64, k: i64, qs: *mut c_void,
                            d: *mut u16, stream: dial_stream) -> dial_status;
    pub fn dial_gguf_unpack(qs: *const c_void, d: *const u16, ty: dial_ggml_type, n: i64, k: i64,
                            blocks: *mut c_void, stream: dial_stream) -> dial_status;
    pub fn dial_gguf_quantize(w: *const f32, ty: dial_ggml_type, n: i64, k: i64, qs: *mut c_void,
                              d: *mut u16, stream: dial_stream) -> dial_status;
    pub fn dial_gguf_dequantize(qs: *const c_void, d: *const u16, ty: dial_ggml_type, n: i64, k: i64,
                                w: *mut c_void, wdt: dial_dtype, stream: dial_stream) -> dial_status;
    pub fn dial_gguf_linear_workspace_bytes(m: i64, k: i64, n: i64) -> usize;
    pub fn dial_gguf_linear(x: *const c_void, xdt: dial_dtype, qs: *const c_void, d: *const u16,
                            ty: dial_ggml_type, y: *mut c_void, m: i64, k: i64, n: i64,
                            workspace: *mut c_void, workspace_bytes: usize,
                            stream: dial_stream) -> dial_status;
    pub fn dial_gguf_linear_noalloc(x: *const c_void, xdt: dial_dtype, qs: *const c_void, d: *const u16,
                                    ty: dial_ggml_type, y: *mut c_void, m: i64, k: i64, n: i64,
                                    stream: dial_stream) -> dial_status;

    // GGUF Q4_K / Q6_K
    pub fn dial_gguf_k_row_bytes(ty: dial_ggml_type, k: i64) -> usize;
    pub fn dial_gguf_k_dequantize(blocks: *const c_void, ty: dial_ggml_type, n: i64, k: i64,
                                  w: *mut c_void, wdt: dial_dtype, stream: dial_stream) -> dial_status;
    pub fn dial_gguf_k_linear(x: *const c_void, xdt: dial_dtype, blocks: *const c_void, ty: dial_ggml_type,
                              y: *mut c_void, m: i64, k: i64, n: i64, stream: dial_stream) -> dial_status;

    // decoder glue (text.rs:1478-1688, llama3/cache.rs:24-217)
    pub fn dial_rmsnorm(x: *const c_void, residual: *const c_void, h_out: *mut c_void, w: *const c_void,
                        y: *mut c_void, dt: dial_dtype, rows: i64, dim: i64, eps: f32,
                        stream: dial_stream) -> dial_status;
    pub fn dial_rope_tables(cos_t: *mut c_void, sin_t: *mut c_void, dt: dial_dtype, max_pos: i64,
                            head_dim: c_int, theta: f32, stream: dial_stream) -> dial_status;
    pub fn dial_qk_norm_rope_kv_append(qkv: *const c_void, q_norm_w: *const c_void, k_norm_w: *const c_void,
                                       cos_t: *const c_void, sin_t: *const c_void, positions: *const i32,
                                       slots: *const i32, q_out: *mut c_void, k_cache: *mut c_void,
                                       v_cache: *mut c_void, dt: dial_dtype, tokens: i64, n_heads: c_int,
                                       n_kv_heads: c_int, head_dim: c_int, max_seq: i64, eps: f32,
                                       qk_norm: c_int, stream: dial_stream) -> dial_status;
    pub fn dial_attention_workspace_bytes(tokens: i64, n_heads: c_int, max_len: i64) -> usize;
    pub fn dial_attention(q: *const c_void, k_cache: *const c_void, v_cache: *const c_void,
                          positions: *const i32, slots: *const i32, out: *mut c_void, workspace: *mut c_void,
                          workspace_bytes: usize, dt: dial_dtype, tokens: i64, n_heads: c_int,
                          n_kv_heads: c_int, head_dim: c_int, max_seq: i64, max_len: i64,
                          stream: dial_stream) -> dial_status;
    pub fn dial_decode_attention_workspace_bytes(n_heads: c_int, max_len: i64) -> usize;
    pub fn dial_decode_attention(qkv: *const c_void, q_norm_w: *const c_void, k_norm_w: *const c_void,
                                 cos_t: *const c_void, sin_t: *const c_void, positions: *const i32,
                                 slots: *const i32, k_cache: *mut c_void, v_cache: *mut c_void,
                                 out: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
                                 dt: dial_dtype, n_heads: c_int, n_kv_heads: c_int, head_dim: c_int,
                                 max_seq: i64, max_len: i64, eps: f32, qk_norm: c_int,
                                 stream: dial_stream) -> dial_status;
    pub fn dial_swiglu(gate_up: *const c_void, out: *mut c_void, dt: dial_dtype, tokens: i64,
                       intermediate: i64, stream: dial_stream) -> dial_status;
    pub fn dial_embedding(table: *const c_void, ids: *const i32, out: *mut c_void, dt: dial_dtype, tokens: i64,
                          vocab: i64, dim: i64, stream: dial_stream) -> dial_status;
    pub fn dial_argmax(x: *const c_void, out: *mut i32, dt: dial_dtype, rows: i64, n: i64,
                       stream: dial_stream) -> dial_status;

    // decoder stage (Transformer::forward text.rs:1636-1688; head qwen3_vl.rs:2420-2451)
    pub fn dial_decoder_workspace_bytes(dims: *const dial_decoder_dims, tokens: i64, max_len: i64) -> usize;
    pub fn dial_decoder_layers(dims: *const dial_decoder_dims, layers: *const dial_layer_weights,
                               n_layers: c_int, hidden: *mut c_void, positions: *const i32, slots: *const i32,
                               tokens: i64, max_len: i64, cos_t: *const c_void, sin_t: *const c_void,
                               workspace: *mut c_void, workspace_bytes: usize,
                               stream: dial_stream) -> dial_status;
    pub fn dial_decoder_head(dims: *const dial_decoder_dims, final_norm: *const c_void, head: dial_linear_ref,
                             hidden: *const c_void, row_index: *const i32, rows: i64, out_ids: *mut i32,
                             logits: *mut c_void, workspace: *mut c_void, workspace_bytes: usize,
                             stream: dial_stream) -> dial_status;
    pub fn dial_decoder_head_shard(dims: *const dial_decoder_dims, final_norm: *const c_void,
                                   head_shard: dial_linear_ref, vocab_offset: i64, shard_rows: i64,
                                   hidden: *const c_void, row_index: *const i32, rows: i64,
                                   out_keys: *mut u64, logits: *mut c_void, workspace: *mut c_void,
                                   workspace_bytes: usize, stream: dial_stream) -> dial_status;
    pub fn dial_head_merge(keys: *const u64, n_shards: c_int, rows: i64, out_ids: *mut i32,
                           stream: dial_stream) -> dial_status;

    // stage planner (AutoPlanner::plan_with_algorithm, spm/planner.rs:378-522)
    pub fn dial_plan_stages(model: *const dial_plan_model, objective: *const dial_plan_objective,
                            devices: *const dial_plan_device, n_devices: c_int, algorithm: c_int,
                            out: *mut dial_plan_result) -> dial_status;

    // stage hand-off over NCCL (RawTensor + TCP, spm/proto/message.rs:147-408, spm/worker.rs:645-765)
    pub fn dial_stage_comm_unique_id(id_out: *mut u8) -> dial_status;
    pub fn dial_stage_comm_init(unique_id: *const u8, rank: c_int, nranks: c_int, device: c_int,
                                timeout_s: f64, out: *mut *mut dial_stage_comm) -> dial_status;
    pub fn dial_stage_comm_send(comm: *mut dial_stage_comm, buf: *const c_void, bytes: usize, peer: c_int,
                                stream: dial_stream) -> dial_status;
    pub fn dial_stage_comm_recv(comm: *mut dial_stage_comm, buf: *mut c_void, bytes: usize, peer: c_int,
                                stream: dial_stream) -> dial_status;
    pub fn dial_stage_comm_wait(comm: *mut dial_stage_comm, stream: dial_stream) -> dial_status;
    pub fn dial_stage_comm_destroy(comm: *mut dial_stage_comm) -> dial_status;
}

// ------------------------------------------------------------------ safe layer

/// A failed call: its status and the library's message for it.
#[derive(Clone, Debug, PartialEq, Eq)]
pub struct Error {
    pub status: dial_status,
    pub message: String,
}

impl std::fmt::Display for Error {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "dial_cuda status {}: {}", self.status, self.message)
    }
}

impl std::error::Error for Error {}

pub type Result<T> = std::result::Result<T, Error>;

/// The calling thread's message for the last failure ("" if none).
pub fn last_error() -> String {
    // SAFETY: the library returns a pointer to a NUL-terminated thread-local buffer.
    unsafe { CStr::from_ptr(dial_last_error()).to_string_lossy().into_owned() }
}

/// Maps a status to `Result`, taking the message from `dial_last_error`.
pub fn check(status: dial_status) -> Result<()> {
    if status == DIAL_OK {
        Ok(())
    } else {
        Err(Error { status, message: last_error() })
    }
}

/// Device pointers of a W8A16 linear (int8 [N, K] row-major + scale [N]).
#[derive(Clone, Copy, Debug)]
pub struct W8A16Weights {
    pub q: *const i8,
    pub scale: *const c_void,
    pub scale_dtype: dial_dtype,
    pub out_dim: i64,
    pub in_dim: i64,
}

/// `CudaW8A16Linear::forward` (worker_w8a16.rs:368-386): y [rows, N] = x [rows, K] . W^T,
/// f16/bf16 activations, on `stream`, with a caller-owned workspace of
/// `dial_w8a16_linear_workspace_bytes(N)` bytes (zero-filled before first use).
///
/// # Safety
/// Every pointer must be a live device allocation of the stated size on the
/// stream's device; `y` must not alias `x`.
pub unsafe fn w8a16_linear(w: &W8A16Weights, x: *const c_void, xdt: dial_dtype, y: *mut c_void, rows: i64,
                           workspace: *mut c_void, workspace_bytes: usize, stream: dial_stream) -> Result<()> {
    check(dial_w8a16_linear(x, xdt, w.q, w.scale, w.scale_dtype, y, rows, w.in_dim, w.out_dim, workspace,
                            workspace_bytes, stream))
}

/// Device pointers of a GGUF Q4_0 / Q8_0 linear in the repacked layout.
#[derive(Clone, Copy, Debug)]
pub struct GgufWeights {
    pub qs: *const c_void,
    pub d: *const u16,
    pub ty: dial_ggml_type,
    pub out_dim: i64,
    pub in_dim: i64,
}

/// `forward_worker_gguf` (worker_gguf.rs:574-611): y keeps x's dtype.
///
/// # Safety
/// As for `w8a16_linear`; the workspace holds
/// `dial_gguf_linear_workspace_bytes(rows, K, N)` bytes, zero-filled before first use.
pub unsafe fn gguf_linear(w: &GgufWeights, x: *const c_void, xdt: dial_dtype, y: *mut c_void, rows: i64,
                          workspace: *mut c_void, workspace_bytes: usize, stream: dial_stream) -> Result<()> {
    check(dial_gguf_linear(x, xdt, w.qs, w.d, w.ty, y, rows, w.in_dim, w.out_dim, workspace, workspace_bytes,
                           stream))
}

/// One pipeline link over NCCL; freed (bounded) on drop.
pub struct StageComm {
    raw: *mut dial_stage_comm,
}

impl StageComm {
    /// A clique id for a new link, made by its sender and shared out of band.
    pub fn unique_id() -> Result<[u8; DIAL_STAGE_COMM_ID_BYTES]> {
        let mut id = [0u8; DIAL_STAGE_COMM_ID_BYTES];
        // SAFETY: `id` holds DIAL_STAGE_COMM_ID_BYTES bytes.
        check(unsafe { dial_stage_comm_unique_id(id.as_mut_ptr()) })?;
        Ok(id)
    }

    /// Joins the link as `rank` of `nranks` on `device`; bounded by `timeout_s`.
    pub fn new(id: &[u8; DIAL_STAGE_COMM_ID_BYTES], rank: i32, nranks: i32, device: i32,
               timeout_s: f64) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        // SAFETY: `id` is a full clique id and `raw` an out-pointer.
        check(unsafe { dial_stage_comm_init(id.as_ptr(), rank, nranks, device, timeout_s, &mut raw) })?;
        Ok(StageComm { raw })
    }

    /// Enqueues a send of `bytes` of device memory to `peer` on `stream`.
    ///
    /// # Safety
    /// `buf` must stay valid until the stream has run the transfer.
    pub unsafe fn send(&self, buf: *const c_void, bytes: usize, peer: i32, stream: dial_stream) -> Result<()> {
        check(dial_stage_comm_send(self.raw, buf, bytes, peer, stream))
    }

    /// Enqueues a receive of `bytes` into device memory from `peer` on `stream`.
    ///
    /// # Safety
    /// `buf` must stay valid and unread until the stream has run the transfer.
    pub unsafe fn recv(&self, buf: *mut c_void, bytes: usize, peer: i32, stream: dial_stream) -> Result<()> {
        check(dial_stage_comm_recv(self.raw, buf, bytes, peer, stream))
    }

    /// Bounded host wait until `stream` is idle.
    pub fn wait(&self, stream: dial_stream) -> Result<()> {
        // SAFETY: the communicator is live.
        check(unsafe { dial_stage_comm_wait(self.raw, stream) })
    }
}

impl Drop for StageComm {
    fn drop(&mut self) {
        // SAFETY: `raw` came from dial_stage_comm_init and is freed once.
        unsafe {
            dial_stage_comm_destroy(self.raw);
        }
    }
}
