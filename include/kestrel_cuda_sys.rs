//! kestrel-cuda-sys: Rust declarations of the C ABI in `kestrel_cuda.h`
//! (libkestrel_cuda.so, the B200 MoE FFN path), one to one, for Kestrel
//! (edition 2021, rust-version 1.87). As a crate this file is `src/lib.rs`;
//! its build script points the linker at the library's directory:
//!
//! ```text
//! println!("cargo:rustc-link-search=native={}", env!("KESTREL_CUDA_LIB_DIR"));
//! ```
//!
//! Every function returns a status (`KC_OK` or a `KC_ERR_*` code) unless its
//! return type says otherwise; the message of the last failure is
//! `kc_last_error(ctx)` (ctx may be null for `kc_init`'s errors). Pointers
//! are host memory for the plain calls and device memory for the `_dev`
//! calls and `kc_route_noalloc`; the library copies what it keeps.
#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_int, c_void, CStr};

/// One context per GPU (`kc_init` / `kc_free`).
#[repr(C)]
pub struct kc_ctx {
    _p: [u8; 0],
}

// status codes
pub const KC_OK: c_int = 0;
pub const KC_ERR_ARG: c_int = 1;
pub const KC_ERR_SHAPE: c_int = 2;
pub const KC_ERR_TYPE: c_int = 3;
pub const KC_ERR_CUDA: c_int = 4;
pub const KC_ERR_NCCL: c_int = 5;
pub const KC_ERR_TIMEOUT: c_int = 6;
pub const KC_ERR_STATE: c_int = 7;
pub const KC_ERR_OOM: c_int = 8;

// ggml tensor types
pub const KC_F32: c_int = 0;
pub const KC_Q8_0: c_int = 8;
pub const KC_Q4_K: c_int = 12;
pub const KC_Q6_K: c_int = 14;

// expert cache policies
pub const KC_EXPERT_POLICY_LFRU: c_int = 0;
pub const KC_EXPERT_POLICY_LRU: c_int = 1;

// kc_expert_cache_stats fields (KC_XS_N of them)
pub const KC_XS_CAPACITY: c_int = 0;
pub const KC_XS_CACHED: c_int = 1;
pub const KC_XS_REQUESTS: c_int = 2;
pub const KC_XS_HITS: c_int = 3;
pub const KC_XS_LATE: c_int = 4;
pub const KC_XS_MISSES: c_int = 5;
pub const KC_XS_SCRATCH_LOADS: c_int = 6;
pub const KC_XS_BYTES_READ: c_int = 7;
pub const KC_XS_PREFETCH_ISSUED: c_int = 8;
pub const KC_XS_PREFETCH_USED: c_int = 9;
pub const KC_XS_PREFETCH_WASTED: c_int = 10;
pub const KC_XS_EVICTIONS: c_int = 11;
pub const KC_XS_LOOKAHEAD_PREDICTED: c_int = 12;
pub const KC_XS_LOOKAHEAD_CORRECT: c_int = 13;
pub const KC_XS_READS: c_int = 14;
pub const KC_XS_FORCED: c_int = 15;
pub const KC_XS_SCRATCH: c_int = 16;
pub const KC_XS_SPEC: c_int = 17;
pub const KC_XS_SPEC_PAUSES: c_int = 18;
pub const KC_XS_N: c_int = 19;

// kc_profile_read stages
pub const KC_STAGE_ROUTER_LOGITS: c_int = 0;
pub const KC_STAGE_ROUTE: c_int = 1;
pub const KC_STAGE_DISPATCH: c_int = 2;
pub const KC_STAGE_QUANT_X: c_int = 3;
pub const KC_STAGE_GATE_UP_INT8: c_int = 4;
pub const KC_STAGE_GATE_UP_F32: c_int = 5;
pub const KC_STAGE_QUANT_ACT: c_int = 6;
pub const KC_STAGE_DOWN_INT8: c_int = 7;
pub const KC_STAGE_DOWN_F32: c_int = 8;
pub const KC_STAGE_COMBINE: c_int = 9;
pub const KC_STAGE_EXPERT_LOAD: c_int = 10;
pub const KC_N_STAGES: c_int = 11;

// kc_set_option options
pub const KC_OPT_F32_PREFILL: c_int = 1;
pub const KC_OPT_LOOKAHEAD: c_int = 2;

// model architectures
pub const KC_ARCH_LLAMA: c_int = 0;
pub const KC_ARCH_QWEN2: c_int = 1;
pub const KC_ARCH_QWEN3: c_int = 2;

// per-layer model tensors (kc_model_tensor kind)
pub const KC_T_ATTN_NORM: c_int = 0;
pub const KC_T_ATTN_Q: c_int = 1;
pub const KC_T_ATTN_K: c_int = 2;
pub const KC_T_ATTN_V: c_int = 3;
pub const KC_T_ATTN_OUT: c_int = 4;
pub const KC_T_ATTN_Q_BIAS: c_int = 5;
pub const KC_T_ATTN_K_BIAS: c_int = 6;
pub const KC_T_ATTN_V_BIAS: c_int = 7;
pub const KC_T_ATTN_Q_NORM: c_int = 8;
pub const KC_T_ATTN_K_NORM: c_int = 9;
pub const KC_T_FFN_NORM: c_int = 10;
pub const KC_T_FFN_GATE: c_int = 11;
pub const KC_T_FFN_UP: c_int = 12;
pub const KC_T_FFN_DOWN: c_int = 13;

// whole-model tensors (kc_model_tensor with layer -1)
pub const KC_T_TOKEN_EMBD: c_int = 0;
pub const KC_T_OUTPUT_NORM: c_int = 1;
pub const KC_T_OUTPUT: c_int = 2;

#[link(name = "kestrel_cuda")]
unsafe extern "C" {
    // context, streams and workspace
    pub fn kc_init(device: c_int, out: *mut *mut kc_ctx) -> c_int;
    pub fn kc_free(ctx: *mut kc_ctx);
    pub fn kc_last_error(ctx: *const kc_ctx) -> *const c_char;
    pub fn kc_set_stream(ctx: *mut kc_ctx, cuda_stream: *mut c_void) -> c_int;
    pub fn kc_reserve(ctx: *mut kc_ctx, max_tokens: c_int) -> c_int;
    pub fn kc_sync(ctx: *mut kc_ctx) -> c_int;
    pub fn kc_device_bytes(ctx: *const kc_ctx) -> i64;
    pub fn kc_set_option(ctx: *mut kc_ctx, option: c_int, value: c_int) -> c_int;
    // weights (HBM-resident expert table, router, dense tensors)
    pub fn kc_upload_experts(ctx: *mut kc_ctx, layer: c_int, n_expert: c_int, d: c_int, ff: c_int,
        t_gate: c_int, gate: *const c_void, t_up: c_int, up: *const c_void, t_down: c_int,
        down: *const c_void, src_on_device: c_int) -> c_int;
    pub fn kc_upload_experts_range(ctx: *mut kc_ctx, layer: c_int, n_expert: c_int, first_expert: c_int,
        n_local: c_int, d: c_int, ff: c_int, t_gate: c_int, gate: *const c_void, t_up: c_int,
        up: *const c_void, t_down: c_int, down: *const c_void, src_on_device: c_int) -> c_int;
    pub fn kc_upload_router(ctx: *mut kc_ctx, layer: c_int, router_w: *const f32, n_expert: c_int, d: c_int,
        k: c_int, norm_topk: c_int, weights_scale: f32, src_on_device: c_int) -> c_int;
    pub fn kc_upload_dense(ctx: *mut kc_ctx, tensor_id: c_int, t: c_int, w: *const c_void, rows: i64,
        cols: i64, src_on_device: c_int) -> c_int;
    pub fn kc_upload_shared_expert(ctx: *mut kc_ctx, layer: c_int, ff_shared: c_int, d: c_int, t_gate: c_int,
        gate: *const c_void, t_up: c_int, up: *const c_void, t_down: c_int, down: *const c_void,
        gate_inp: *const f32, src_on_device: c_int) -> c_int;
    // host-streamed experts
    pub fn kc_upload_experts_streamed(ctx: *mut kc_ctx, layer: c_int, n_expert: c_int, d: c_int, ff: c_int,
        t_gate: c_int, gate: *const c_void, t_up: c_int, up: *const c_void, t_down: c_int,
        down: *const c_void, src_on_device: c_int) -> c_int;
    pub fn kc_expert_cache_reserve(ctx: *mut kc_ctx, capacity: c_int, scratch: c_int, spec: c_int,
        policy: c_int) -> c_int;
    pub fn kc_expert_prefetch(ctx: *mut kc_ctx, layer: c_int, experts: *const i32, n: c_int) -> c_int;
    pub fn kc_expert_cache_stats(ctx: *const kc_ctx, out: *mut u64, n: c_int) -> c_int; // KC_XS_* fields
    pub fn kc_expert_cache_decay(ctx: *mut kc_ctx) -> c_int;
    // the hot path: Transformer::moe_ffn and quant::matmul
    pub fn kc_moe_ffn(ctx: *mut kc_ctx, layer: c_int, h: *const f32, n_tok: c_int, router_w: *const f32,
        n_expert: c_int, k: c_int, norm_topk: c_int, weights_scale: f32, out: *mut f32, topk_ids: *mut i32,
        topk_w: *mut f32) -> c_int;
    pub fn kc_moe_ffn_dev(ctx: *mut kc_ctx, layer: c_int, h: *const f32, n_tok: c_int, out: *mut f32,
        topk_ids: *mut i32, topk_w: *mut f32) -> c_int;
    pub fn kc_matmul(ctx: *mut kc_ctx, tensor_id: c_int, x: *const f32, n: c_int, out: *mut f32) -> c_int;
    pub fn kc_matmul_dev(ctx: *mut kc_ctx, tensor_id: c_int, x: *const f32, n: c_int, out: *mut f32) -> c_int;
    // building blocks on device buffers (the context's stream)
    pub fn kc_q8k_quantize_dev(ctx: *mut kc_ctx, x: *const f32, n_rows: i64, cols: i64, q: *mut i8,
        d: *mut f32, bsums: *mut i32) -> c_int;
    pub fn kc_q8_quantize_dev(ctx: *mut kc_ctx, x: *const f32, n_rows: i64, cols: i64, q: *mut i8,
        d: *mut f32, s16: *mut i32) -> c_int;
    pub fn kc_route_dev(ctx: *mut kc_ctx, logits: *const f32, n_tok: c_int, n_expert: c_int, k: c_int,
        norm_topk: c_int, weights_scale: f32, ids: *mut i32, w: *mut f32) -> c_int;
    pub fn kc_router_logits_dev(ctx: *mut kc_ctx, router_w: *const f32, n_expert: c_int, d: c_int,
        h: *const f32, n_tok: c_int, logits: *mut f32) -> c_int;
    pub fn kc_block_sums_dev(ctx: *mut kc_ctx, t: c_int, w: *const c_void, rows: i64, cols: i64, q: *const i8,
        bsums: *const i32, n_act: c_int, out: *mut i32) -> c_int;
    pub fn kc_quantize_dev(ctx: *mut kc_ctx, t: c_int, x: *const f32, rows: i64, cols: i64,
        out: *mut c_void) -> c_int;
    // measurement
    pub fn kc_profile_enable(ctx: *mut kc_ctx, on: c_int) -> c_int;
    pub fn kc_profile_read(ctx: *mut kc_ctx, stage_ms: *mut f64, stage_calls: *mut i64,
        n_stages: c_int) -> c_int;
    pub fn kc_kernel_launches() -> i64;
    // routing without device allocation (device pointers, caller's stream)
    pub fn kc_route_noalloc(router_w: *const f32, n_expert: c_int, d: c_int, h: *const f32, n_tok: c_int,
        k: c_int, norm_topk: c_int, weights_scale: f32, topk_ids: *mut i32, topk_w: *mut f32,
        stream: *mut c_void) -> c_int;
    // whole-model decode
    pub fn kc_model_init(ctx: *mut kc_ctx, n_layer: c_int, d: c_int, n_head: c_int, n_head_kv: c_int,
        head_dim: c_int, n_vocab: c_int, n_ctx: c_int, rope_dim: c_int, rope_base: f32, rms_eps: f32,
        arch: c_int) -> c_int;
    pub fn kc_model_tensor(ctx: *mut kc_ctx, layer: c_int, kind: c_int, t: c_int, w: *const c_void, rows: i64,
        cols: i64, src_on_device: c_int) -> c_int;
    pub fn kc_model_forward(ctx: *mut kc_ctx, tokens: *const u32, n: c_int, logits: *mut f32,
        next_token: *mut u32) -> c_int;
    pub fn kc_model_generate(ctx: *mut kc_ctx, prompt: *const u32, n_prompt: c_int, n_gen: c_int,
        out_tokens: *mut u32) -> c_int;
    pub fn kc_model_set_sequences(ctx: *mut kc_ctx, n_seq: c_int) -> c_int;
    pub fn kc_model_prefill_seq(ctx: *mut kc_ctx, seq: c_int, prompt: *const u32, n: c_int,
        next_token: *mut u32) -> c_int;
    pub fn kc_model_decode_seqs(ctx: *mut kc_ctx, n_seq: c_int, n_gen: c_int, out_tokens: *mut u32) -> c_int;
    pub fn kc_model_generate_batch(ctx: *mut kc_ctx, n_seq: c_int, prompts: *const u32,
        prompt_lens: *const c_int, n_gen: c_int, out_tokens: *mut u32) -> c_int;
    pub fn kc_model_truncate(ctx: *mut kc_ctx, keep: c_int) -> c_int;
    pub fn kc_model_cached(ctx: *const kc_ctx) -> c_int;
    // GGUF / KGUF loading
    pub fn kc_load_gguf(ctx: *mut kc_ctx, path: *const c_char, n_ctx: c_int, info_json: *mut c_char,
        cap: i64) -> c_int;
    pub fn kc_gguf_inspect(path: *const c_char, out: *mut c_char, cap: i64) -> c_int;
    // expert parallelism (one process per GPU)
    pub fn kc_ep_unique_id(out: *mut c_char) -> c_int; // out: 128 bytes
    pub fn kc_ep_init(ctx: *mut kc_ctx, rank: c_int, world: c_int, uid: *const c_char) -> c_int; // uid: 128 bytes
    pub fn kc_ep_reserve(ctx: *mut kc_ctx, max_tokens: c_int) -> c_int;
}

/// Error text of the last failed call (ctx may be null for kc_init errors).
pub fn last_error(ctx: *const kc_ctx) -> String {
    unsafe { CStr::from_ptr(kc_last_error(ctx)).to_string_lossy().into_owned() }
}
