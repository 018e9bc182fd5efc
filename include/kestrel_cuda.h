/*
 * kestrel_cuda.h -- C ABI of the B200 (sm_100a) MoE FFN backend for Kestrel.
 *
 * The boundary a Kestrel host (Rust `extern "C"` crate, C++ or Python ctypes)
 * crosses to run the Mixture-of-Experts FFN hot path on an NVIDIA B200. Plain
 * pointers and sizes only; every entry point returns a kc_status (0 = OK) and
 * never unwinds across the ABI. The message of the last failure is available
 * from kc_last_error(). Reference interfaces replaced (paths are relative to
 * the Kestrel repository, Eduardo7125/kestrel):
 *
 *   kc_init / kc_free        NativeSession::load's engine set-up
 *                            (crates/kestrel-backends/src/lib.rs:125-187)
 *   kc_upload_experts        ExpertStore::preload_all + ExpertBuf::part
 *                            (crates/kestrel-memory/src/expert.rs:620-641, 62-76)
 *   kc_upload_experts_streamed / kc_expert_cache_reserve / kc_expert_prefetch /
 *   kc_expert_cache_stats / kc_expert_cache_decay
 *                            ExpertStore::new / request / get / prefetch /
 *                            metrics / decay (expert.rs:223-551) with HBM
 *                            slots as the cache
 *   kc_upload_router         the router tensor ffn_gate_inp.weight read through
 *                            Lease::tensor (crates/kestrel-memory/src/store.rs:233)
 *   kc_upload_dense          WeightStore::lease + Lease::tensor for a dense weight
 *                            (crates/kestrel-memory/src/store.rs:233-244, 400-470)
 *   kc_moe_ffn[_dev]         Transformer::moe_ffn with Transformer::route inside
 *                            (crates/kestrel-engine/src/transformer.rs:513-589, 472-496)
 *   kc_matmul[_dev]          quant::matmul (crates/kestrel-engine/src/quant.rs:229-339)
 *   kc_q8k_quantize_dev      Q8KRow::quantize (crates/kestrel-engine/src/qdot.rs:347-367)
 *   kc_q8_quantize_dev       Q8Row::quantize (crates/kestrel-engine/src/qdot.rs:29-49)
 *   kc_route_dev             Transformer::route (transformer.rs:472-496)
 *   kc_block_sums_dev        the per-superblock integer sums of avx2::dot_q4_k_8k /
 *                            dot_q6_k_8k (crates/kestrel-engine/src/avx2.rs:351-419)
 *   kc_last_error            EngineError's message (transformer.rs:15-27)
 *   kc_model_init / _tensor  Transformer::new's weight lookup and KV cache
 *                            (crates/kestrel-engine/src/transformer.rs:147-272)
 *   kc_model_forward         Transformer::forward (transformer.rs:280-302, 375-467)
 *   kc_model_generate        the greedy loop of Engine::generate with
 *                            SamplerConfig::greedy (crates/kestrel-engine/src/
 *                            lib.rs:116-145, sampler.rs:25-27, 104-112)
 *   kc_model_truncate        Transformer::truncate (transformer.rs:276-278)
 *   kc_model_set_sequences / _prefill_seq / _decode_seqs / _generate_batch
 *                            n independent Engine::generate greedy loops
 *                            (lib.rs:98-166; the reference serves one sequence
 *                            per Engine) decoded in lockstep on one context
 *
 * Threading: a context is used by one host thread at a time (the reference's
 * Transformer is `&mut self` per forward, transformer.rs:278). One context per
 * GPU; for expert parallelism one process per GPU, each with its own context.
 *
 * `*_dev` entry points take device pointers and enqueue work on the context's
 * stream without synchronising; the others take host pointers, copy in, run,
 * copy out and synchronise.
 */
#ifndef KESTREL_CUDA_H
#define KESTREL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KC_API __attribute__((visibility("default")))
#else
#define KC_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kc_ctx kc_ctx;

/* Status codes. Shapes and types are checked before any work is enqueued. */
enum {
  KC_OK = 0,
  KC_ERR_ARG = 1,     /* null pointer, bad layer/tensor id, bad option      */
  KC_ERR_SHAPE = 2,   /* dimension not supported (block multiple, limits)   */
  KC_ERR_TYPE = 3,    /* ggml type without a CUDA kernel                    */
  KC_ERR_CUDA = 4,    /* a CUDA runtime call failed                         */
  KC_ERR_NCCL = 5,    /* an NCCL call failed                                */
  KC_ERR_TIMEOUT = 6, /* a kernel's bounded wait expired (device status)    */
  KC_ERR_STATE = 7,   /* call out of order (e.g. layer not uploaded)        */
  KC_ERR_OOM = 8      /* device allocation failed                           */
};

/* ggml type ids (crates/kestrel-gguf/src/types.rs:48-86) with CUDA kernels. */
enum { KC_F32 = 0, KC_Q8_0 = 8, KC_Q4_K = 12, KC_Q6_K = 14 };

/* ---- context ------------------------------------------------------------ */

/* Create a context on CUDA device `device` with its own stream. */
KC_API int kc_init(int device, kc_ctx** out);
/* Free all memory owned by the context: device weights and workspace, and the
   pinned host memory of host-streamed experts. Waits for its work first. */
KC_API void kc_free(kc_ctx* ctx);
/* Message of the last failed call on this context ("" if none). ctx may be
   NULL for errors of kc_init. */
KC_API const char* kc_last_error(const kc_ctx* ctx);
/* Enqueue subsequent work on a caller-owned cudaStream_t (NULL = the legacy
   default stream). The context's own stream is used until this is called. */
KC_API int kc_set_stream(kc_ctx* ctx, void* cuda_stream);
/* Size the workspace for up to `max_tokens` tokens per call (grows on demand
   otherwise; call before capturing a CUDA graph). */
KC_API int kc_reserve(kc_ctx* ctx, int max_tokens);
/* Wait for all work on the context's stream; reports kernel timeouts. */
KC_API int kc_sync(kc_ctx* ctx);
/* Bytes of device memory held by the context (weights + workspace). */
KC_API int64_t kc_device_bytes(const kc_ctx* ctx);

/* ---- weights (HBM-resident expert table) ---------------------------------
   Expert tensors are GGUF "stacked" tensors: expert e's gate/up rows start at
   e * ff * bytes_for(t, d) and its down rows at e * d * bytes_for(t, ff)
   (TensorInfo::slice_offset, crates/kestrel-gguf/src/lib.rs:183-189).
   `src_on_device` = 1 when the pointers are device memory (e.g. weights made
   on the GPU), 0 for host memory. The bytes are converted once into the
   device layout the kernels read; the caller's buffers are not kept. */
KC_API int kc_upload_experts(kc_ctx* ctx, int layer, int n_expert, int d, int ff, int t_gate, const void* gate,
                      int t_up, const void* up, int t_down, const void* down, int src_on_device);
/* Upload a subset of a layer's experts: stacked tensors holding `n_local`
   experts whose global ids are first_expert .. first_expert+n_local-1
   (expert-parallel sharding). */
KC_API int kc_upload_experts_range(kc_ctx* ctx, int layer, int n_expert, int first_expert, int n_local, int d, int ff,
                            int t_gate, const void* gate, int t_up, const void* up, int t_down, const void* down,
                            int src_on_device);
/* Router weights ffn_gate_inp.weight, F32 [n_expert, d], and the MoeInfo
   routing options (crates/kestrel-model/src/lib.rs:103-117): top-k, whether
   the selected weights are renormalised, and weights_scale (0 or 1 = none). */
KC_API int kc_upload_router(kc_ctx* ctx, int layer, const float* router_w, int n_expert, int d, int k, int norm_topk,
                     float weights_scale, int src_on_device);
/* A dense weight [rows, cols] of type `t` addressed by `tensor_id`. */
KC_API int kc_upload_dense(kc_ctx* ctx, int tensor_id, int t, const void* w, int64_t rows, int64_t cols,
                    int src_on_device);

/* Shared expert of layer `layer` (qwen2moe: ffn_{gate,up,down}_shexp.weight,
   read at crates/kestrel-engine/src/transformer.rs:188-191): gate / up
   [ff_shared, d], down [d, ff_shared], and the optional F32 gate vector
   ffn_gate_inp_shexp.weight [d] (NULL: gate 1). kc_moe_ffn then adds, after
   the routed experts, out[s] += sigmoid(gate_inp . h[s]) *
   down(SwiGLU(gate h[s], up h[s])) as Transformer::moe_ffn does
   (transformer.rs:571-587). d % 256 == 0, ff_shared % 32 == 0. */
KC_API int kc_upload_shared_expert(kc_ctx* ctx, int layer, int ff_shared, int d, int t_gate, const void* gate,
                                   int t_up, const void* up, int t_down, const void* down, const float* gate_inp,
                                   int src_on_device);

/* ---- host-streamed experts (models larger than HBM) ----------------------
   ExpertStore's expert cache (crates/kestrel-memory/src/expert.rs:305-551)
   with HBM as the cache and pinned host memory as the backing store, for
   models whose experts do not all fit on the GPU.

   kc_upload_experts_streamed takes the same arguments as kc_upload_experts
   (ExpertStore::new's per-layer tensors, expert.rs:223) but keeps the
   converted experts in pinned host memory. Every kc_moe_ffn* call of such a
   layer routes on the GPU, reads the routed ids back (one synchronisation),
   copies the experts it routes to that are not resident into HBM slots
   (ExpertStore::request + get, expert.rs:358-424, 523-537: hits, misses,
   evictions by the LFRU or LRU score of expert.rs:305-331) and computes the
   same results, bit for bit, as the resident layer. A call's experts are
   resident all at once: capacity + scratch must be at least the number of
   distinct experts one call routes to. Calls of streamed layers cannot be
   captured into a CUDA graph (kc_model_generate then runs its steps
   eagerly). Every streamed layer has the same shape (d, ff, types). Not
   available with expert parallelism. A call or prefetch whose expert copy
   CUDA refuses returns KC_ERR_CUDA after emptying the cache (the copies
   already queued land first), so no slot counts as holding an expert whose
   copy did not run; the counters are reset with it.

   kc_expert_cache_reserve sets `capacity` cache slots, `scratch` slots for
   experts the cache does not admit, `spec` slots for predictions it does
   not admit (ExpertStore::new's capacity, scratch_slots and spec_slots) and
   the policy; until it is called a context holds one layer's experts
   (capacity n_expert, no scratch or spec slots, LFRU). It forgets what the
   slots held and resets the counters.

   kc_expert_prefetch is ExpertStore::prefetch (expert.rs:451-521): starts
   copying experts of `layer` that are not resident, on a copy stream, into
   cache slots when the cache admits them, else into the speculative slots
   (replacing the oldest landed guess; paused for 4096 predictions when
   fewer than half of the last 128 were used); never waits. The whole-model path (kc_model_*)
   calls it itself, as the router lookahead of transformer.rs:432-436,
   498-508 does: for steps of at most 4 rows, the next streamed layer's
   experts are predicted from the current post-attention state
   (KC_OPT_LOOKAHEAD, on by default).

   kc_expert_cache_stats writes up to n counters (ExpertMetrics,
   expert.rs:127-153), indexed by KC_XS_*. kc_expert_cache_decay halves the
   experts' heat (ExpertStore::decay, expert.rs:545-551). */
enum { KC_EXPERT_POLICY_LFRU = 0, KC_EXPERT_POLICY_LRU = 1 };
enum {
  KC_XS_CAPACITY = 0,
  KC_XS_CACHED = 1,
  KC_XS_REQUESTS = 2,
  KC_XS_HITS = 3,
  KC_XS_LATE = 4,            /* resident but its prefetch copy still landing */
  KC_XS_MISSES = 5,
  KC_XS_SCRATCH_LOADS = 6,
  KC_XS_BYTES_READ = 7,      /* bytes copied host -> HBM                      */
  KC_XS_PREFETCH_ISSUED = 8,
  KC_XS_PREFETCH_USED = 9,
  KC_XS_PREFETCH_WASTED = 10,
  KC_XS_EVICTIONS = 11,
  KC_XS_LOOKAHEAD_PREDICTED = 12,
  KC_XS_LOOKAHEAD_CORRECT = 13,
  KC_XS_READS = 14,          /* host -> HBM copies issued                     */
  KC_XS_FORCED = 15,         /* admitted without the policy's consent: scratch slots exhausted */
  KC_XS_SCRATCH = 16,
  KC_XS_SPEC = 17,
  KC_XS_SPEC_PAUSES = 18,    /* speculative pool paused for low accuracy     */
  KC_XS_N = 19
};
KC_API int kc_upload_experts_streamed(kc_ctx* ctx, int layer, int n_expert, int d, int ff, int t_gate,
                                      const void* gate, int t_up, const void* up, int t_down, const void* down,
                                      int src_on_device);
KC_API int kc_expert_cache_reserve(kc_ctx* ctx, int capacity, int scratch, int spec, int policy);
KC_API int kc_expert_prefetch(kc_ctx* ctx, int layer, const int32_t* experts, int n);
KC_API int kc_expert_cache_stats(const kc_ctx* ctx, uint64_t* out, int n);
KC_API int kc_expert_cache_decay(kc_ctx* ctx);

/* ---- hot path ----------------------------------------------------------- */

/* Transformer::moe_ffn for `layer`: h [n_tok, d] f32 -> out [n_tok, d] f32.
   router_w may be NULL (use the uploaded router); otherwise it is a host F32
   [E, d] matrix used for this call with the given k / norm_topk /
   weights_scale. topk_ids [n_tok, k] / topk_w [n_tok, k] are optional outputs
   (NULL to skip) in the reference's order (descending probability). Host
   buffers; synchronous. */
KC_API int kc_moe_ffn(kc_ctx* ctx, int layer, const float* h, int n_tok, const float* router_w, int n_expert, int k,
               int norm_topk, float weights_scale, float* out, int32_t* topk_ids, float* topk_w);
/* Same on device buffers, enqueued on the context stream (uploaded router). */
KC_API int kc_moe_ffn_dev(kc_ctx* ctx, int layer, const float* h, int n_tok, float* out, int32_t* topk_ids,
                   float* topk_w);

/* quant::matmul for an uploaded dense tensor: x [n, cols] f32 -> out [n, rows]
   f32, with the reference's dispatch on n. F32 tensors: the reference's f32
   summation order, bit-exact, for every n. n < 4: int8 activations for
   Q4_K/Q6_K/Q8_0, bit-exact. n >= 4: the reference's dequantise-then-f32
   path, run on tcgen05 tensor cores with f16 operands and f32 accumulation
   (within 1e-3 of the output's scale), or exactly in f32 on CUDA cores under
   KC_OPT_F32_PREFILL. */
KC_API int kc_matmul(kc_ctx* ctx, int tensor_id, const float* x, int n, float* out);
KC_API int kc_matmul_dev(kc_ctx* ctx, int tensor_id, const float* x, int n, float* out);

/* ---- building blocks on device buffers (tests, custom pipelines) ------- */

/* Q8KRow::quantize of n_rows rows of `cols` floats (cols % 256 == 0):
   q [n_rows, cols] int8, d [n_rows, cols/256] f32, bsums [n_rows, cols/16]. */
KC_API int kc_q8k_quantize_dev(kc_ctx* ctx, const float* x, int64_t n_rows, int64_t cols, int8_t* q, float* d,
                        int32_t* bsums);
/* Q8Row::quantize (cols % 32 == 0): d [n_rows, cols/32], s16 [n_rows, cols/16]. */
KC_API int kc_q8_quantize_dev(kc_ctx* ctx, const float* x, int64_t n_rows, int64_t cols, int8_t* q, float* d,
                       int32_t* s16);
/* Transformer::route on precomputed logits [n_tok, E]. */
KC_API int kc_route_dev(kc_ctx* ctx, const float* logits, int n_tok, int n_expert, int k, int norm_topk,
                 float weights_scale, int32_t* ids, float* w);
/* Router logits with the reference's exact operation order (quant::matmul of
   an F32 [E, d] weight): h [n_tok, d] -> logits [n_tok, E]. */
KC_API int kc_router_logits_dev(kc_ctx* ctx, const float* router_w, int n_expert, int d, const float* h, int n_tok,
                         float* logits);
/* Per-superblock integer sums of a GGUF K-quant matrix [rows, cols] (raw GGUF
   bytes on the device) against Q8_K activation rows: out [n_act, rows,
   cols/256, 9] int32 = the eight 32-bit lanes of sumi and the min (Q4_K) or
   offset (Q6_K) term of avx2::dot_q4_k_8k / dot_q6_k_8k. */
KC_API int kc_block_sums_dev(kc_ctx* ctx, int t, const void* w, int64_t rows, int64_t cols, const int8_t* q,
                      const int32_t* bsums, int n_act, int32_t* out);
/* This library's deterministic quantizer (same rules as the Python one):
   x [rows, cols] f32 -> GGUF bytes [rows, bytes_for(t, cols)]. */
KC_API int kc_quantize_dev(kc_ctx* ctx, int t, const float* x, int64_t rows, int64_t cols, void* out);

/* ---- profiling ---------------------------------------------------------
   When enabled, kc_moe_ffn* records a CUDA event pair around each stage of
   the layer on the context stream; kc_profile_read synchronises, returns the
   milliseconds and call counts accumulated per stage since the previous read,
   and resets them. Stage ids: */
enum {
  KC_STAGE_ROUTER_LOGITS = 0,
  KC_STAGE_ROUTE = 1,
  KC_STAGE_DISPATCH = 2,
  KC_STAGE_QUANT_X = 3,
  KC_STAGE_GATE_UP_INT8 = 4,
  KC_STAGE_GATE_UP_F32 = 5,
  KC_STAGE_QUANT_ACT = 6,
  KC_STAGE_DOWN_INT8 = 7,
  KC_STAGE_DOWN_F32 = 8,
  KC_STAGE_COMBINE = 9,
  KC_STAGE_EXPERT_LOAD = 10, /* host-streamed layers: ids read back, expert copies */
  KC_N_STAGES = 11
};
KC_API int kc_profile_enable(kc_ctx* ctx, int on);
KC_API int kc_profile_read(kc_ctx* ctx, double* stage_ms, int64_t* stage_calls, int n_stages);
/* Number of CUDA kernels this library has launched in the process so far
   (all contexts and threads; graph replays count each captured kernel once,
   at capture). A caller reads it before and after a run to count the
   launches the run made. No counterpart in Kestrel (a measurement hook). */
KC_API int64_t kc_kernel_launches(void);

/* ---- routing without device allocation ----------------------------------
   No counterpart in Kestrel: an addition for hosts that cannot let a library
   allocate device memory -- a session whose memory ledger must account for
   every byte, a latency-critical decode thread that cannot afford the
   device-wide synchronisation cudaMalloc/cudaFree may cause, or an embedding
   that hands out device memory only from its own pool. Computes what kc_router_logits_dev followed by
   kc_route_dev compute (router logits in the reference's operation order,
   softmax, top-k, optional renormalisation and weights_scale) on device
   buffers, enqueued on `stream` (NULL = legacy default stream), with no
   cudaMalloc/cudaFree: the logits live in a fixed array compiled into the
   library (65536 floats, 256 KB, held on every GPU that loads the library
   until the process exits). Needs no context; errors are read with
   kc_last_error(NULL).
   Limits: n_tok * n_expert <= 65536 (larger requests return KC_ERR_SHAPE);
   1 <= k <= min(64, n_expert); n_expert <= 1024.
   The first call on each device looks up the array's device address; make
   that first call before capturing a stream. All calls on a device share the
   one array: calls whose kernels may overlap on the GPU (different streams
   without ordering) race, so serialise them.
   The call returns once its kernels are enqueued. If one of its bounded
   device-side waits expires (a GPU stalled for seconds), every selection of
   the call is written as id -1 with weight 0: a caller that cannot rule this
   out checks the ids for -1 after synchronising the stream. */
KC_API int kc_route_noalloc(const float* router_w, int n_expert, int d, const float* h, int n_tok, int k,
                            int norm_topk, float weights_scale, int32_t* topk_ids, float* topk_w, void* stream);

/* ---- options ------------------------------------------------------------ */
enum {
  /* value 1: products with n >= 4 rows (prefill) run on CUDA cores in f32 on
     exactly dequantised weights, as quant::matmul's gemm_f32 path does,
     instead of tcgen05 with f16 operands (0, the default). */
  KC_OPT_F32_PREFILL = 1,
  /* value 1 (default): the whole-model path predicts the next host-streamed
     layer's experts and prefetches them (router lookahead); 0: off. */
  KC_OPT_LOOKAHEAD = 2
};
KC_API int kc_set_option(kc_ctx* ctx, int option, int value);

/* ---- whole model: the dense decode path around the MoE layers ----------
   Transformer::forward for llama / qwen2 / qwen3 and their MoE variants:
   embedding rows (quant::get_row), per layer RMSNorm, q/k/v projections
   (+ biases for qwen2, q/k RMSNorm for qwen3), RoPE (interleaved for llama,
   NeoX otherwise; angles from the C library's powf/sinf/cosf), an f16 KV
   cache of n_ctx positions, causal GQA attention, the output projection, the
   FFN and the residuals; then the final norm, the output head (the embedding
   when no output tensor is given) and argmax. Routed layers use the experts,
   router and shared expert uploaded with kc_upload_experts /
   kc_upload_router / kc_upload_shared_expert under the same layer index;
   other layers need KC_T_FFN_GATE/UP/DOWN. Prompts are processed in chunks of
   256 tokens (Transformer::n_batch). */
enum { KC_ARCH_LLAMA = 0, KC_ARCH_QWEN2 = 1, KC_ARCH_QWEN3 = 2 };
/* Tensor kinds of a layer (GGUF blk.N.*). Norms and biases are F32 vectors;
   the matrices are quantized [rows, cols] with GGUF's row-major bytes. */
enum {
  KC_T_ATTN_NORM = 0,   /* attn_norm.weight [d]                          */
  KC_T_ATTN_Q = 1,      /* attn_q.weight [n_head * head_dim, d]          */
  KC_T_ATTN_K = 2,      /* attn_k.weight [n_head_kv * head_dim, d]       */
  KC_T_ATTN_V = 3,      /* attn_v.weight [n_head_kv * head_dim, d]       */
  KC_T_ATTN_OUT = 4,    /* attn_output.weight [d, n_head * head_dim]     */
  KC_T_ATTN_Q_BIAS = 5, /* attn_q.bias (qwen2)                           */
  KC_T_ATTN_K_BIAS = 6,
  KC_T_ATTN_V_BIAS = 7,
  KC_T_ATTN_Q_NORM = 8, /* attn_q_norm.weight [head_dim] (qwen3)         */
  KC_T_ATTN_K_NORM = 9,
  KC_T_FFN_NORM = 10,   /* ffn_norm.weight [d]                           */
  KC_T_FFN_GATE = 11,   /* dense FFN: ffn_gate / ffn_up [n_ff, d]        */
  KC_T_FFN_UP = 12,
  KC_T_FFN_DOWN = 13    /* ffn_down [d, n_ff]                            */
};
/* Model tensors (layer = -1). */
enum { KC_T_TOKEN_EMBD = 0, KC_T_OUTPUT_NORM = 1, KC_T_OUTPUT = 2 };

/* Declare the model. Replaces a previous model, its KV cache and the routed
   layers uploaded under indices 0 .. n_layer-1: upload the new model's
   experts and routers after this call. */
KC_API int kc_model_init(kc_ctx* ctx, int n_layer, int d, int n_head, int n_head_kv, int head_dim, int n_vocab,
                         int n_ctx, int rope_dim, float rope_base, float rms_eps, int arch);
KC_API int kc_model_tensor(kc_ctx* ctx, int layer, int kind, int t, const void* w, int64_t rows, int64_t cols,
                           int src_on_device);
/* Feed n tokens after the cached ones; logits [n_vocab] of the last token
   and/or its argmax (either may be NULL). Host buffers; synchronous. */
KC_API int kc_model_forward(kc_ctx* ctx, const uint32_t* tokens, int n, float* logits, uint32_t* next_token);
/* Greedy decode: forward the prompt, then n_gen tokens, each step's argmax
   fed to the next step from device memory (no host round trip per token).
   out_tokens [n_gen]. */
KC_API int kc_model_generate(kc_ctx* ctx, const uint32_t* prompt, int n_prompt, int n_gen, uint32_t* out_tokens);
/* Several independent sequences on one context, each with its own KV cache
   (sequence 0's is the one the calls above use), decoded in lockstep.
   kc_model_set_sequences: room for n_seq (1..32) sequences; growing it drops
   every cached position (KC_ERR_OOM if the caches do not fit).
   kc_model_prefill_seq: evaluate a prompt alone in sequence `seq`'s cache,
   from position 0; its greedy next token (also returned, may be NULL) becomes
   the sequence's pending token.
   kc_model_decode_seqs: n_gen greedy tokens of each of sequences 0..n_seq-1,
   one row per sequence per step, each row computed as a batch of one would be
   (router in quant::dot order, int8 products), so sequence s gets exactly the
   tokens kc_model_generate gives for its prompt alone. out_tokens
   [n_seq][n_gen]; column 0 is the pending token, and the last token becomes
   the new pending one (a later call continues). n_seq * top-k <= 1024.
   kc_model_forward, _generate and _truncate on sequence 0 leave it without a
   pending token.
   kc_model_generate_batch: the three in one call (prompts concatenated in
   `prompts`, prompt_lens[s] tokens each). */
KC_API int kc_model_set_sequences(kc_ctx* ctx, int n_seq);
KC_API int kc_model_prefill_seq(kc_ctx* ctx, int seq, const uint32_t* prompt, int n, uint32_t* next_token);
KC_API int kc_model_decode_seqs(kc_ctx* ctx, int n_seq, int n_gen, uint32_t* out_tokens);
KC_API int kc_model_generate_batch(kc_ctx* ctx, int n_seq, const uint32_t* prompts, const int* prompt_lens,
                                   int n_gen, uint32_t* out_tokens);
/* Forget cached positions from `keep` on; kc_model_cached = positions held. */
KC_API int kc_model_truncate(kc_ctx* ctx, int keep);
KC_API int kc_model_cached(const kc_ctx* ctx);

/* ---- model files -----------------------------------------------------------
   GGUF v2/v3 and Kestrel-prepared KGUF containers (GgufFile::open,
   crates/kestrel-gguf/src/lib.rs:196-311; strided expert slices read at
   TensorInfo::slice_offset, lib.rs:183-189). Hyper-parameters as kestrel-model
   reads them (crates/kestrel-model/src/lib.rs:170-215, 338-373). */

/* Declare the file's model on the context (kc_model_init) and upload every
   tensor Transformer::new reads (transformer.rs:147-213): the dense ones
   through kc_model_tensor, routed experts, router and shared expert through
   kc_upload_experts / kc_upload_router / kc_upload_shared_expert -- the
   HBM-resident expert table in place of ExpertStore::preload_all
   (NativeSession::load, crates/kestrel-backends/src/lib.rs:133-157). Before
   uploading anything, the device bytes of the weights, the f16 KV cache for
   n_ctx positions and a workspace allowance are checked against the GPU's
   free memory: a model that does not fit returns KC_ERR_OOM (the VRAM tier
   of the planner's placement decision, crates/kestrel-planner/src/
   lib.rs:429-439). info_json (optional, cap bytes) receives a JSON summary.
   Types with kernels: F32, Q8_0, Q4_K, Q6_K; others return KC_ERR_TYPE. */
KC_API int kc_load_gguf(kc_ctx* ctx, const char* path, int n_ctx, char* info_json, int64_t cap);
/* Parse a GGUF / KGUF file without a GPU or a context: a JSON description
   (version, alignment, derived hyper-parameters, tensors with file offsets,
   sizes and strides) into out (cap bytes). Errors: kc_last_error(NULL). */
KC_API int kc_gguf_inspect(const char* path, char* out, int64_t cap);

/* ---- expert parallelism (one process per GPU, NCCL over NVLink) -------- */

/* 128-byte NCCL unique id, created on one rank and shared by the host. */
KC_API int kc_ep_unique_id(char out[128]);
/* Join an expert-parallel group of `world` ranks; experts of every layer are
   owned by rank e / (E / world) (contiguous blocks). */
KC_API int kc_ep_init(kc_ctx* ctx, int rank, int world, const char uid[128]);
/* Map every rank's exchange arena over NVLink (CUDA IPC) for up to
   `max_tokens` tokens per rank and kc_moe_ffn call (collective; call after
   uploading the layers and routers, on every rank). Calls within that
   capacity then exchange token rows and result rows with this library's own
   kernels through peer memory, with no host synchronisation; larger calls use
   NCCL. The path is chosen per call from the rank's own token count, so in
   each call every rank must be on the same side of max_tokens (as when all
   ranks serve batches of one size); otherwise the ranks on different paths
   wait for each other until the bounded waits expire (KC_ERR_TIMEOUT). */
KC_API int kc_ep_reserve(kc_ctx* ctx, int max_tokens);

#ifdef __cplusplus
}
#endif

#endif /* KESTREL_CUDA_H */
