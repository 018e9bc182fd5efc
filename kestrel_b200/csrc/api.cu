// C ABI of the B200 MoE FFN backend (include/kestrel_cuda.h): the context, the
// HBM-resident expert table, the workspace and the layer pipeline
//   router logits -> route (top-k) -> dispatch (permute metadata)
//   -> gate/up (+SwiGLU) -> down -> combine (un-permute)
// behind Transformer::moe_ffn / quant::matmul's call surface.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "decode.h"
#include "expert_cache.h"
#include "ep.h"
#include "kernels.h"
#include "mma.h"
#include "loader.h"
#include "model.h"

using namespace kc;

namespace {

struct Layer {
  // Routed experts: expert e (global id) lives at (e - first_expert) in the
  // stacked device buffers.
  bool has_experts = false;
  int id = -1;  // layer index
  int n_expert = 0, first_expert = 0, n_local = 0, d = 0, ff = 0;
  int t_gate = 0, t_up = 0, t_down = 0;
  int64_t mb_gate = 0, mb_down = 0;  // device bytes of one expert's gate (= up) / down matrix
  uint8_t* gate = nullptr;
  uint8_t* up = nullptr;
  uint8_t* down = nullptr;
  // Host-streamed experts (kc_upload_experts_streamed): every expert's gate,
  // up and down in the device layout, one pinned host block of slot_bytes per
  // expert ([gate | up | down] at 0, up_off, down_off), copied per call into
  // the context's HBM slots. `slot` is set only on the per-call copy of the
  // layer that the kernels see (expert e at slot[e]).
  bool streamed = false;
  uint8_t* host = nullptr;
  int64_t slot_bytes = 0, up_off = 0, down_off = 0;
  const int* slot = nullptr;
  // Router (ffn_gate_inp.weight) and MoeInfo options.
  bool has_router = false;
  float* router = nullptr;
  int k = 0, norm_topk = 1;
  float weights_scale = 0.f;
  // Shared expert (qwen2moe): dense gate/up [sh_ff, d], down [d, sh_ff],
  // optional F32 gate vector [d].
  bool has_shared = false;
  int sh_ff = 0;
  struct Mat {
    int t = 0;
    int64_t rows = 0, cols = 0;
    uint8_t* w = nullptr;
  } sh_gate, sh_up, sh_down;
  float* sh_inp = nullptr;
};

struct Dense {
  int t = 0;
  int64_t rows = 0, cols = 0, rs = 0;  // rs: F32 row stride (bytes)
  uint8_t* w = nullptr;
};

// Workspace sized by (tokens, experts, k, d, ff); carved from one allocation.
struct Work {
  int T = 0, E = 0, K = 0, D = 0, F = 0;
  void* arena = nullptr;
  size_t bytes = 0;
  float* logits = nullptr;
  int* ids = nullptr;
  float* w = nullptr;
  int8_t* xq = nullptr;
  float* xd = nullptr;
  int32_t* xs = nullptr;
  uint8_t* xrec = nullptr;  // activation records of the input rows
  DispatchOut meta{};
  float* g = nullptr;       // gate / up outputs per slot
  float* u = nullptr;
  uint8_t* arec = nullptr;  // activation records of SwiGLU(g, u) per slot
  float* act = nullptr;
  __half* x16 = nullptr;    // f16 input rows per slot (tensor-core path)
  __half* act16 = nullptr;  // f16 SwiGLU rows per slot
  int8_t* aq = nullptr;
  float* ad = nullptr;
  int32_t* as = nullptr;
  float* y = nullptr;
  float* h_in = nullptr;   // staging for host-pointer calls
  float* out = nullptr;
  float* router_tmp = nullptr;
  float* mma_part = nullptr;  // split-K partial tiles of the tcgen05 kernel
  int* mma_cnt = nullptr;     // its per-tile counters (zeroed at allocation)
  // Metadata of a dense product of dmeta_n rows (one group), kept apart from
  // the MoE dispatch so that repeated products with the same n reuse it.
  DispatchOut dmeta{};
  int dmeta_n = -1;
  // Tensor maps of the f16 activation rows (tcgen05 B operand), encoded once
  // per (buffer, rows, cols): x16 for gate/up and dense products, act16 for
  // down.
  struct MapCache {
    const void* ptr = nullptr;
    int64_t rows = -1, cols = -1;
    MmaMaps maps;
  } map_x16, map_act16;
};

// Expert-parallel exchange buffers. Home side (this rank's tokens): routing,
// plans, the rows sent and the result rows received. Owner side (rows received
// from every rank): the rows, their selections and the result rows sent back.
struct EpBufs {
  int T = 0, k = 0, d = 0;  // home capacity: tokens, selections, d
  int* ids_home = nullptr;
  float* w_home = nullptr;
  int* send_tok = nullptr;  // [world][T]
  int* ret_pos = nullptr;   // [T * k]
  int* xch = nullptr;       // [2][world][2]: counts sent, counts received
  float* sendbuf = nullptr; // [world * T][d]
  int32_t* sendmeta = nullptr;
  float* retrecv = nullptr; // [T * k][d]
  int R = 0, RS = 0;        // owner capacity: received rows, result rows sent
  float* recvbuf = nullptr;
  int32_t* recvmeta = nullptr;
  int* ids_loc = nullptr;
  float* w_loc = nullptr;
  int* ret_send_pos = nullptr;
  float* retsend = nullptr;
  int* xch_host = nullptr;  // pinned copy of xch
};

}  // namespace

// Per-stage CUDA event pairs (kc_profile_enable).
struct Prof {
  bool on = false;
  struct Rec {
    int stage;
    cudaEvent_t a, b;
  };
  std::vector<cudaEvent_t> pool;
  std::vector<Rec> recs;
  cudaEvent_t take() {
    if (pool.empty()) {
      cudaEvent_t e;
      cudaEventCreate(&e);
      return e;
    }
    cudaEvent_t e = pool.back();
    pool.pop_back();
    return e;
  }
};

struct Model;  // the dense decode path of a whole model (kc_model_*)

// Host-streamed experts (kc_upload_experts_streamed): the HBM slots a call's
// experts are copied into, their bookkeeping (expert_cache.h), and the
// buffers of the per-call slot table and the routed ids read back to the host.
struct ExpertStreams {
  ExpertCache cache;
  int capacity = -1, scratch = 0, spec = 0;  // slots; capacity -1: not reserved (default at first use)
  ExpertPolicy policy = ExpertPolicy::Lfru;
  int64_t slot_bytes = 0;          // one expert's [gate | up | down]; shared by every streamed layer
  uint8_t* arena = nullptr;        // [capacity + scratch + spec][slot_bytes]
  int* slot_dev = nullptr;         // slot table of the current call, [table_e]
  int* slot_host = nullptr;        // its pinned source
  int table_e = 0;
  int32_t* ids_host = nullptr;     // pinned: a call's routed ids, then the lookahead's
  int ids_cap = 0;
  cudaStream_t copy = nullptr;     // prefetch copies
  std::vector<cudaEvent_t> ready;  // per slot: its latest prefetch copy
  int n_layers = 0;                // streamed layers uploaded
  bool lookahead = true;           // KC_OPT_LOOKAHEAD
  // Lookahead predictions awaiting their layer's call (recall counters).
  std::map<int, std::vector<int>> predicted;
  // A lookahead's ids on the device (written on the auxiliary stream), read
  // back at the next demand synchronisation.
  int look_layer = -1;
  const int32_t* look_ids = nullptr;
  int look_n = 0;
};

struct kc_ctx {
  int device = 0;
  // n >= 4 products on CUDA cores in f32 instead of tcgen05 with f16
  // operands (KC_OPT_F32_PREFILL).
  bool f32_prefill = false;
  // Every row as a batch of one (independent sequences decoded in lockstep):
  // router sums in quant::dot order, every expert and dense product on the
  // int8 path in entries of at most three rows. Set only inside
  // kc_model_decode_seqs's steps.
  bool rows_mode = false;
  Model* model = nullptr;
  // Auxiliary stream for the n >= 4 products that run beside the int8 ones,
  // and the fork / join events (created on first use).
  cudaStream_t aux = nullptr;
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
  // Stream on which decode steps are captured as a graph (the context stream
  // may be the legacy default stream, which cannot be captured).
  cudaStream_t cap = nullptr;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  int* status = nullptr;  // device word written by kernels on timeout
  int* status_host = nullptr;  // pinned host copy of it (check_status)
  std::string err;
  std::map<int, Layer> layers;
  std::map<int, Dense> dense;
  Work ws;
  Work ws_ep;  // the owner-side expert products of expert parallelism
  int64_t weight_bytes = 0;
  ExpertStreams xs;
  EpState ep;
  EpBufs epb;
  Prof prof;
};

namespace {
// Brackets one pipeline stage with an event pair when profiling is on.
struct StageScope {
  kc_ctx* c;
  Prof::Rec r{};
  StageScope(kc_ctx* ctx, int stage) : c(ctx) {
    if (!c->prof.on) return;
    r.stage = stage;
    r.a = c->prof.take();
    r.b = c->prof.take();
    cudaEventRecord(r.a, c->stream);
  }
  ~StageScope() {
    if (!c->prof.on) return;
    cudaEventRecord(r.b, c->stream);
    c->prof.recs.push_back(r);
  }
};
}  // namespace

namespace {

thread_local std::string g_init_err;

int fail(kc_ctx* c, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (c) c->err = buf;
  else g_init_err = buf;
  return code;
}

#define CK(call)                                                                         \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return fail(ctx, e_ == cudaErrorMemoryAllocation ? KC_ERR_OOM : KC_ERR_CUDA,       \
                  "%s failed: %s", #call, cudaGetErrorString(e_));                       \
  } while (0)

#define CKL()                                                                            \
  do {                                                                                   \
    cudaError_t e_ = cudaGetLastError();                                                 \
    if (e_ != cudaSuccess)                                                               \
      return fail(ctx, KC_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e_)); \
  } while (0)

#define RC(call)                                \
  do {                                          \
    int r_ = (call);                            \
    if (r_ != KC_OK) {                          \
      if (ctx->err.empty()) ctx->err = #call;   \
      return r_;                                \
    }                                           \
  } while (0)

bool type_ok(int t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q8_0; }
bool is_k(int t) { return t == T_Q4_K || t == T_Q6_K; }

size_t al(size_t v) { return (v + 255) & ~size_t(255); }
// Bytes of the activation records of one slot of `cols` values (the larger of
// the Q8_K and Q8 formats).
size_t rec_bytes(int64_t cols) {
  return (size_t)std::max(rec_row_bytes(true, cols), rec_row_bytes(false, cols)) + 512;
}

// (Re)allocate workspace w so it holds at least the given dimensions.
int ensure_work(kc_ctx* ctx, Work& w, int T, int E, int K, int D, int F) {
  if (T <= w.T && E <= w.E && K <= w.K && D <= w.D && F <= w.F && w.arena) return KC_OK;
  T = std::max(T, w.T);
  E = std::max(E, w.E);
  K = std::max(K, w.K);
  D = std::max(D, w.D);
  F = std::max(F, w.F);
  T = std::max(T, 1);
  E = std::max(E, 1);
  K = std::max(K, 1);
  D = std::max(D, 256);
  F = std::max(F, 256);
  const size_t A = (size_t)T * K;
  std::vector<size_t> sz = {
      (size_t)T * E * 4,                 // logits
      A * 4, A * 4,                      // ids, w
      (size_t)T * D, (size_t)T * (D / 32 + 1) * 4, (size_t)T * (D / 16 + 1) * 4,  // xq xd xs
      A * rec_bytes(D),                  // xrec
      (size_t)E * 4, (size_t)(E + 1) * 4, A * 4, A * 4, A * 4, std::max((size_t)E, A) * 4, (size_t)E * 4, 16,  // meta
      (size_t)(E + 1) * 4,               // large_tt
      A * F * 4, A * F * 4,              // g, u
      A * rec_bytes(F),                  // arec
      A * F * 4,                         // act
      A * D * 2, A * F * 2,              // x16, act16
      A * F, A * (F / 32 + 1) * 4, A * (F / 16 + 1) * 4,  // aq ad as
      A * D * 4,                         // y
      (size_t)T * D * 4, (size_t)T * D * 4,  // h_in, out
      (size_t)E * D * 4,                 // router_tmp
      mma_part_bytes(), mma_cnt_bytes(),  // mma_part, mma_cnt
      64, 64, 64, 64, 64, 64,             // dmeta: counts, offsets, small, large, n_lists, large_tt
  };
  size_t total = 0;
  for (size_t s : sz) total += al(s);
  if (w.arena) {
    CK(cudaStreamSynchronize(ctx->stream));
    CK(cudaFree(w.arena));
    w.arena = nullptr;
  }
  CK(cudaMalloc(&w.arena, total));
  w.bytes = total;
  w.T = T; w.E = E; w.K = K; w.D = D; w.F = F;
  char* p = static_cast<char*>(w.arena);
  size_t i = 0;
  auto take = [&](void** dst) {
    *dst = p;
    p += al(sz[i++]);
  };
  take((void**)&w.logits);
  take((void**)&w.ids);
  take((void**)&w.w);
  take((void**)&w.xq);
  take((void**)&w.xd);
  take((void**)&w.xs);
  take((void**)&w.xrec);
  take((void**)&w.meta.counts);
  take((void**)&w.meta.offsets);
  take((void**)&w.meta.slot_tok);
  take((void**)&w.meta.slot_w);
  take((void**)&w.meta.tok_slot);
  take((void**)&w.meta.small_list);
  take((void**)&w.meta.large_list);
  take((void**)&w.meta.n_lists);
  take((void**)&w.meta.large_tt);
  take((void**)&w.g);
  take((void**)&w.u);
  take((void**)&w.arec);
  take((void**)&w.act);
  take((void**)&w.x16);
  take((void**)&w.act16);
  take((void**)&w.aq);
  take((void**)&w.ad);
  take((void**)&w.as);
  take((void**)&w.y);
  take((void**)&w.h_in);
  take((void**)&w.out);
  take((void**)&w.router_tmp);
  take((void**)&w.mma_part);
  take((void**)&w.mma_cnt);
  take((void**)&w.dmeta.counts);
  take((void**)&w.dmeta.offsets);
  take((void**)&w.dmeta.small_list);
  take((void**)&w.dmeta.large_list);
  take((void**)&w.dmeta.n_lists);
  take((void**)&w.dmeta.large_tt);
  w.dmeta_n = -1;
  CK(cudaMemsetAsync(w.mma_cnt, 0, mma_cnt_bytes(), ctx->stream));
  return KC_OK;
}
int ensure_work(kc_ctx* ctx, int T, int E, int K, int D, int F) { return ensure_work(ctx, ctx->ws, T, E, K, D, F); }

// Waits for the context stream and reads the kernels' status word (one
// stream-ordered copy into pinned memory, then one synchronisation).
int check_status(kc_ctx* ctx) {
  CK(cudaMemcpyAsync(ctx->status_host, ctx->status, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));
  const int st = *ctx->status_host;
  if (st != 0) {
    // Cleared on the context's stream (non-blocking: a legacy-stream memset
    // would not be ordered before the next call's kernels, whose bounded
    // waits read the word and return early on KC_ERR_STATE).
    CK(cudaMemsetAsync(ctx->status, 0, sizeof(int), ctx->stream));
    CK(cudaStreamSynchronize(ctx->stream));
    static const char* sites[] = {"unknown", "decode producer (empty stage)", "decode consumer (full stage)",
                                  "decode drain", "tcgen05 producer (raw stage)", "tcgen05 producer (operand stage)",
                                  "tcgen05 producer drain", "tcgen05 MMA issuer (operand stage)",
                                  "tcgen05 MMA issuer (accumulator)", "tcgen05 dequantiser (raw stage)",
                                  "tcgen05 dequantiser (operand stage)", "tcgen05 epilogue (accumulator)",
                                  "router logits (bulk copy)", "tcgen05 MMA issuer drain",
                                  "decode consumer (previous lap of a stage)",
                                  "expert-parallel peer exchange (another rank did not publish)",
                                  "expert-parallel exchange (the ranks chose different paths, peer memory "
                                  "and NCCL, in one call: every rank must be on the same side of the "
                                  "kc_ep_reserve capacity)",
                                  "tcgen05 producer (a slot tile larger than the launch's bound)"};
    const int site = st >> 8;
    return fail(ctx, st & 0xFF, "a kernel's bounded wait expired (status %d) at: %s", st & 0xFF,
                site >= 0 && site < (int)(sizeof(sites) / sizeof(sites[0])) ? sites[site] : "unknown");
  }
  return KC_OK;
}

// Convert `n_mats` stacked GGUF matrices [rows, cols] (host or device bytes)
// into the device layout at dst.
int upload_matrix(kc_ctx* ctx, int t, const void* src, int64_t n_mats, int64_t rows, int64_t cols, uint8_t* dst,
                  bool on_dev) {
  const int64_t mat_src = rows * gguf_row_bytes(t, cols), mat_dst = dev_matrix_bytes(t, rows, cols);
  if (on_dev) {
    RC(launch_repack(t, src, n_mats, rows, cols, dst, ctx->stream));
    CKL();
    return KC_OK;
  }
  // Host source: stage whole matrices through a bounded device buffer.
  const int64_t chunk = std::max<int64_t>(1, (256ll << 20) / std::max<int64_t>(mat_src, 1));
  void* tmp = nullptr;
  CK(cudaMalloc(&tmp, std::min(n_mats, chunk) * mat_src));
  for (int64_t m0 = 0; m0 < n_mats; m0 += chunk) {
    const int64_t nm = std::min(chunk, n_mats - m0);
    cudaError_t e = cudaMemcpyAsync(tmp, static_cast<const uint8_t*>(src) + m0 * mat_src, nm * mat_src,
                                    cudaMemcpyHostToDevice, ctx->stream);
    int rc = e == cudaSuccess ? launch_repack(t, tmp, nm, rows, cols, dst + m0 * mat_dst, ctx->stream) : KC_ERR_CUDA;
    if (rc == KC_OK) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess || rc != KC_OK) {
      cudaFree(tmp);
      return fail(ctx, KC_ERR_CUDA, "upload failed: %s", cudaGetErrorString(e));
    }
  }
  CK(cudaFree(tmp));
  return KC_OK;
}

// Device-memory sources of an upload may still be written by work on another
// stream (e.g. a framework's default stream): wait for the whole device before
// reading them on the context stream.
int wait_device_source(kc_ctx* ctx, bool on_dev) {
  if (on_dev) CK(cudaDeviceSynchronize());
  return KC_OK;
}

int ensure_aux(kc_ctx* ctx) {
  if (ctx->aux) return KC_OK;
  CK(cudaStreamCreateWithFlags(&ctx->aux, cudaStreamNonBlocking));
  CK(cudaEventCreateWithFlags(&ctx->ev_fork, cudaEventDisableTiming));
  CK(cudaEventCreateWithFlags(&ctx->ev_join, cudaEventDisableTiming));
  return KC_OK;
}

GroupedArgs grouped_base(kc_ctx* ctx) {
  GroupedArgs a{};
  a.status = ctx->status;
  return a;
}

// ---- host-streamed experts ---------------------------------------------------
// Experts of a streamed layer live in pinned host memory in the device
// layout; a call copies the ones it routes to that are not resident into HBM
// slots (ExpertStore::request / get, crates/kestrel-memory/src/expert.rs:
// 358-424, 523-537) and the kernels read expert e at slot[e].

void streams_free(kc_ctx* ctx) {
  ExpertStreams& S = ctx->xs;
  if (S.copy) cudaStreamSynchronize(S.copy);
  cudaFree(S.arena);
  cudaFree(S.slot_dev);
  if (S.slot_host) cudaFreeHost(S.slot_host);
  if (S.ids_host) cudaFreeHost(S.ids_host);
  for (cudaEvent_t e : S.ready) cudaEventDestroy(e);
  if (S.copy) cudaStreamDestroy(S.copy);
  S.arena = nullptr;
  S.slot_dev = S.slot_host = nullptr;
  S.ids_host = nullptr;
  S.ids_cap = S.table_e = 0;
  S.ready.clear();
  S.copy = nullptr;
  S.predicted.clear();
  S.look_layer = -1;
  S.look_ids = nullptr;
}

// Forget what the slots hold (a streamed layer was replaced or freed): no
// copy may still land in them and no kernel may still read them.
int streams_invalidate(kc_ctx* ctx) {
  ExpertStreams& S = ctx->xs;
  if (S.copy) CK(cudaStreamSynchronize(S.copy));
  CK(cudaStreamSynchronize(ctx->stream));
  if (S.arena) S.cache.configure(S.capacity, S.scratch, S.spec, S.policy);
  S.predicted.clear();
  S.look_layer = -1;
  S.look_ids = nullptr;
  return KC_OK;
}

// The slot arena for the reserved capacity (default: one layer's experts).
int streams_alloc(kc_ctx* ctx, int n_expert) {
  ExpertStreams& S = ctx->xs;
  if (S.arena) return KC_OK;
  if (S.capacity < 0) {
    S.capacity = n_expert;
    S.scratch = S.spec = 0;
  }
  const int slots = S.capacity + S.scratch + S.spec;
  if (slots < 1) return fail(ctx, KC_ERR_STATE, "host-streamed experts: no slots reserved");
  if (cudaMalloc(&S.arena, (size_t)slots * S.slot_bytes) != cudaSuccess) {
    cudaGetLastError();
    S.arena = nullptr;
    return fail(ctx, KC_ERR_OOM, "host-streamed experts: %d slots of %lld bytes do not fit", slots,
                (long long)S.slot_bytes);
  }
  if (!S.copy) CK(cudaStreamCreateWithFlags(&S.copy, cudaStreamNonBlocking));
  S.ready.resize(slots, nullptr);
  for (cudaEvent_t& e : S.ready)
    if (!e) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  S.cache.configure(S.capacity, S.scratch, S.spec, S.policy);
  return KC_OK;
}

// Prefetch copies that have landed (ExpertBuf's ticket done).
void streams_refresh(ExpertStreams& S) {
  for (int s = 0; s < S.cache.slots(); ++s)
    if (S.cache.pending(s) && cudaEventQuery(S.ready[s]) == cudaSuccess) S.cache.mark_done(s);
  cudaGetLastError();  // cudaErrorNotReady is not an error of the call
}

// ExpertStore::prefetch for `experts` (ascending, unique) of streamed layer
// Lt: copies on the copy stream into cache or speculative slots, each
// recording its slot's event. The policy picks no slot that work in flight
// reads (the latest demand call's experts) or that a copy is still filling.
int streams_prefetch(kc_ctx* ctx, const Layer& Lt, const std::vector<int>& experts) {
  ExpertStreams& S = ctx->xs;
  if (experts.empty()) return KC_OK;
  RC(streams_alloc(ctx, Lt.n_expert));
  streams_refresh(S);
  std::vector<ExpertCache::Load> loads;
  S.cache.prefetch(Lt.id, experts.data(), (int)experts.size(), loads);
  for (const ExpertCache::Load& ld : loads) {
    cudaError_t ce = cudaMemcpyAsync(S.arena + (int64_t)ld.slot * S.slot_bytes,
                                     Lt.host + (int64_t)ld.expert * S.slot_bytes, (size_t)S.slot_bytes,
                                     cudaMemcpyHostToDevice, S.copy);
    if (ce == cudaSuccess) ce = cudaEventRecord(S.ready[ld.slot], S.copy);
    if (ce != cudaSuccess) {
      // The slots of this prefetch count as filled by a copy that may never
      // run (an event that was never recorded reads as complete): forget
      // every slot's contents once the copies already queued have landed.
      cudaStreamSynchronize(S.copy);
      S.cache.configure(S.capacity, S.scratch, S.spec, S.policy);
      return fail(ctx, KC_ERR_CUDA, "host-streamed experts: prefetch copy failed: %s", cudaGetErrorString(ce));
    }
    S.cache.add_bytes((uint64_t)S.slot_bytes, 1);
  }
  return KC_OK;
}

int grow_pinned(kc_ctx* ctx, void** p, int& cap, int need, size_t elem) {
  if (need <= cap) return KC_OK;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  cap = 0;
  CK(cudaHostAlloc(p, std::max<size_t>(64, (size_t)need * elem), cudaHostAllocDefault));
  cap = need;
  return KC_OK;
}

// One call of streamed layer L whose routed ids (A of them) are on the
// device: read them back, make every routed expert resident (demand copies on
// the context stream, waits on prefetches still landing), upload the slot
// table, start the lookahead's prefetch if one is pending, and return in Ls
// the layer as the kernels see it.
int streams_demand(kc_ctx* ctx, const Layer& L, const int32_t* ids_dev, int A, Layer& Ls) {
  ExpertStreams& S = ctx->xs;
  cudaStream_t st = ctx->stream;
  const int E = L.n_expert;
  RC(streams_alloc(ctx, E));
  const int look_n = S.look_ids ? S.look_n : 0;
  RC(grow_pinned(ctx, (void**)&S.ids_host, S.ids_cap, A + look_n, 4));
  if (S.table_e < E) {
    cudaFree(S.slot_dev);
    if (S.slot_host) cudaFreeHost(S.slot_host);
    S.slot_dev = S.slot_host = nullptr;
    S.table_e = 0;
    CK(cudaMalloc(&S.slot_dev, (size_t)E * 4));
    CK(cudaHostAlloc(&S.slot_host, (size_t)E * 4, cudaHostAllocDefault));
    S.table_e = E;
  }
  if (A > 0) CK(cudaMemcpyAsync(S.ids_host, ids_dev, (size_t)A * 4, cudaMemcpyDeviceToHost, st));
  if (look_n) CK(cudaMemcpyAsync(S.ids_host + A, S.look_ids, (size_t)look_n * 4, cudaMemcpyDeviceToHost, ctx->aux));
  // Synchronises: every earlier call's kernels are complete after this, so
  // their slots may be overwritten by this call's copies.
  RC(check_status(ctx));
  if (look_n) CK(cudaStreamSynchronize(ctx->aux));
  streams_refresh(S);
  auto unique_ids = [&](const int32_t* ids, int n, int n_exp) {
    std::vector<char> seen(n_exp, 0);
    for (int i = 0; i < n; ++i)
      if (ids[i] >= 0 && ids[i] < n_exp) seen[ids[i]] = 1;
    std::vector<int> out;
    for (int e = 0; e < n_exp; ++e)
      if (seen[e]) out.push_back(e);
    return out;
  };
  const std::vector<int> need = unique_ids(S.ids_host, A, E);
  auto pi = S.predicted.find(L.id);
  if (pi != S.predicted.end()) {  // Transformer::moe_ffn's recall count (transformer.rs:519-524)
    uint64_t correct = 0;
    for (int e : pi->second) correct += std::binary_search(need.begin(), need.end(), e) ? 1 : 0;
    S.cache.record_lookahead(pi->second.size(), correct);
    S.predicted.erase(pi);
  }
  std::vector<int> slot(need.size());
  std::vector<ExpertCache::Load> loads;
  std::vector<int> waits;
  if (!S.cache.demand(L.id, need.data(), (int)need.size(), slot.data(), loads, waits))
    return fail(ctx, KC_ERR_SHAPE,
                "host-streamed experts: layer %d routes to %d experts, more than the %d cache + %d scratch slots "
                "can hold at once (kc_expert_cache_reserve)",
                L.id, (int)need.size(), S.capacity, S.scratch);
  // The cache now counts this call's experts as resident: if a copy cannot
  // be enqueued, forget every slot's contents before reporting the error.
  cudaError_t ce = cudaSuccess;
  for (int s : waits)
    if (ce == cudaSuccess) ce = cudaStreamWaitEvent(st, S.ready[s], 0);
  for (const ExpertCache::Load& ld : loads) {
    if (ce != cudaSuccess) break;
    ce = cudaMemcpyAsync(S.arena + (int64_t)ld.slot * S.slot_bytes, L.host + (int64_t)ld.expert * S.slot_bytes,
                         (size_t)S.slot_bytes, cudaMemcpyHostToDevice, st);
    if (ce == cudaSuccess) S.cache.add_bytes((uint64_t)S.slot_bytes, 1);
  }
  for (size_t i = 0; i < need.size(); ++i) S.slot_host[need[i]] = slot[i];
  if (ce == cudaSuccess) ce = cudaMemcpyAsync(S.slot_dev, S.slot_host, (size_t)E * 4, cudaMemcpyHostToDevice, st);
  if (ce != cudaSuccess) {
    // Prefetch copies still landing would otherwise race with the next
    // call's copies into the slots the reset frees.
    cudaStreamSynchronize(S.copy);
    S.cache.configure(S.capacity, S.scratch, S.spec, S.policy);
    return fail(ctx, KC_ERR_CUDA, "host-streamed experts: expert copy failed: %s", cudaGetErrorString(ce));
  }
  if (look_n) {
    const int nl = S.look_layer;
    S.look_ids = nullptr;
    S.look_layer = -1;
    auto it = ctx->layers.find(nl);
    if (it != ctx->layers.end() && it->second.streamed) {
      std::vector<int> pred = unique_ids(S.ids_host + A, look_n, it->second.n_expert);
      RC(streams_prefetch(ctx, it->second, pred));
      S.predicted[nl] = std::move(pred);
    }
  }
  Ls = L;
  Ls.gate = S.arena;
  Ls.up = S.arena + L.up_off;
  Ls.down = S.arena + L.down_off;
  Ls.mb_gate = Ls.mb_down = S.slot_bytes;
  Ls.first_expert = 0;
  Ls.slot = S.slot_dev;
  return KC_OK;
}

// Drops a layer's host-streamed experts (its pinned block), if it has them.
int drop_streamed(kc_ctx* ctx, Layer& L) {
  if (!L.streamed) return KC_OK;
  RC(streams_invalidate(ctx));
  cudaFreeHost(L.host);
  L.host = nullptr;
  L.streamed = false;
  L.has_experts = false;
  --ctx->xs.n_layers;
  return KC_OK;
}

// Reads a pending lookahead's ids back now (its layer's predecessor is not
// host-streamed, so no demand synchronisation comes first) and prefetches.
int streams_lookahead_now(kc_ctx* ctx) {
  ExpertStreams& S = ctx->xs;
  if (!S.look_ids) return KC_OK;
  const int nl = S.look_layer, n = S.look_n;
  const int32_t* ids_dev = S.look_ids;
  S.look_ids = nullptr;
  S.look_layer = -1;
  auto it = ctx->layers.find(nl);
  if (it == ctx->layers.end() || !it->second.streamed) return KC_OK;
  RC(grow_pinned(ctx, (void**)&S.ids_host, S.ids_cap, n, 4));
  CK(cudaMemcpyAsync(S.ids_host, ids_dev, (size_t)n * 4, cudaMemcpyDeviceToHost, ctx->aux));
  CK(cudaStreamSynchronize(ctx->aux));
  const int E = it->second.n_expert;
  std::vector<char> seen(E, 0);
  for (int i = 0; i < n; ++i)
    if (S.ids_host[i] >= 0 && S.ids_host[i] < E) seen[S.ids_host[i]] = 1;
  std::vector<int> pred;
  for (int e = 0; e < E; ++e)
    if (seen[e]) pred.push_back(e);
  RC(streams_prefetch(ctx, it->second, pred));
  S.predicted[nl] = std::move(pred);
  return KC_OK;
}

}  // namespace

namespace kc {
// Message returned by kc_last_error(NULL) on this thread (entry points
// without a context).
void set_global_error(const char* msg) { g_init_err = msg ? msg : ""; }

// KESTREL_GRAPHS=0 runs every decode step eagerly.
bool model_graphs_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("KESTREL_GRAPHS");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("KESTREL_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

std::atomic<int64_t> g_kernel_launches{0};

int num_sms() {
  // SM count per device, read once per device (several contexts on different
  // GPUs may share the process and call from different threads).
  static std::atomic<int> sms_of[PerDeviceOnce::kMaxDev] = {};
  int cur = 0;
  if (cudaGetDevice(&cur) != cudaSuccess || cur < 0 || cur >= PerDeviceOnce::kMaxDev) return 1;
  int sms = sms_of[cur].load(std::memory_order_relaxed);
  if (sms <= 0) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cur) != cudaSuccess || sms <= 0) return 1;
    sms_of[cur].store(sms, std::memory_order_relaxed);
  }
  return sms;
}
}  // namespace kc

// ---------------------------------------------------------------------------
// Layer pipeline on device buffers. h/out [n_tok, d]; optional ids/w outputs.
// Expert products of n_rows activation rows h for their k selections ids
// (expert ids in [0, E) of the layer's device table, offset by ebase; -1 or
// out-of-range ids are skipped): dispatch (permute), activation records,
// gate/up (+SwiGLU), down. Leaves y [slot, d] and the dispatch metadata
// (slot of every selection in W.meta.tok_slot) in workspace W, which must be
// sized for (n_rows, E, k, d, ff).
// dispatched / recorded: the dispatch metadata / the input rows' records are
// already in W (route_dispatch_kernel).
// The activation tensor maps of a launch, re-encoded only when the buffer or
// its shape changed since the previous call (a map holds only the address,
// shape and strides, so equal keys give equal maps).
static int cached_tmaps(Work::MapCache& c, const void* ptr, int64_t rows, int64_t cols, const MmaMaps*& out) {
  if (c.ptr != ptr || c.rows != rows || c.cols != cols) {
    c.ptr = nullptr;
    if (make_tmaps_f16(c.maps, ptr, rows, cols) != KC_OK) return KC_ERR_CUDA;
    c.ptr = ptr;
    c.rows = rows;
    c.cols = cols;
  }
  out = &c.maps;
  return KC_OK;
}

static int experts_forward(kc_ctx* ctx, Work& W, const Layer& L, int E, int ebase, const float* h, int n_rows,
                           const int* ids, const float* wts, int k, bool dispatched = false,
                           bool recorded = false) {
  const int d = L.d, ff = L.ff;
  cudaStream_t st = ctx->stream;
  if (n_rows == 0) return KC_OK;
  // 2. dispatch metadata (permute).
  if (!dispatched) {
    StageScope ss(ctx, KC_STAGE_DISPATCH);
    RC(launch_dispatch(ids, wts, n_rows, k, E, W.meta, st, ctx->rows_mode));
    CKL();
  }
  const bool kq_in = is_k(L.t_gate), kq_dn = is_k(L.t_down);
  const int A = n_rows * k;
  // By rows, the int8 list has up to one entry per selection.
  const int max_small = ctx->rows_mode ? A : std::min(E, A);
  // An expert holds at most one row per token, so with fewer than 4 rows no
  // expert reaches the n >= 4 path and its launches are skipped; by rows none
  // ever does.
  const bool any_large = n_rows >= 4 && !ctx->rows_mode;
  const bool mma_gu = !ctx->f32_prefill && mma_supported(L.t_gate, d, 2);
  const bool mma_dn = !ctx->f32_prefill && mma_supported(L.t_down, ff, 1) && ff % 256 == 0;
  const int max_tt = ceil_div(A, kMmaTileN) + std::min(E, A / 4);
  // The int8 (1-3 rows) and n >= 4 launches of a stage are independent. When
  // few experts are expected to reach 4 rows (rows per expert ~ Poisson(A / E)
  // for uniform routing, A / E <= 2), the n >= 4 launch, which is then
  // latency-bound, runs on the auxiliary stream beside the int8 one: the int8
  // kernel leaves it `split` SMs (in proportion to the expected weight bytes
  // of each path, at least 8) and the rest of its grid takes the SMs the int8
  // kernel frees. With more rows per expert both run one after the other on
  // all SMs.
  int split = 0;
  const bool fork = any_large && !ctx->prof.on && (double)A <= 2.0 * E;
  if (fork) {
    RC(ensure_aux(ctx));
    const double lam = (double)A / E, p0 = std::exp(-lam);
    const double f_small = p0 * (lam + lam * lam / 2 + lam * lam * lam / 6), f_large = std::max(0.0, 1 - p0 - f_small);
    const int nsm = num_sms();
    split = std::min(nsm / 2, std::max(8, (int)std::lround(nsm * f_large / std::max(1e-9, f_small + f_large))));
  }
  const int dec_ctas = num_sms() - split;
  auto fork_aux = [&]() -> int {
    CK(cudaEventRecord(ctx->ev_fork, st));
    CK(cudaStreamWaitEvent(ctx->aux, ctx->ev_fork, 0));
    return KC_OK;
  };
  auto join_aux = [&]() -> int {
    CK(cudaEventRecord(ctx->ev_join, ctx->aux));
    CK(cudaStreamWaitEvent(st, ctx->ev_join, 0));
    return KC_OK;
  };
  cudaStream_t lst = fork ? ctx->aux : st;  // stream of the n >= 4 launches
  // 3. activation records of every slot's input row (int8 path) and its f16
  //    copy (tensor-core path).
  if (!recorded) {
    StageScope ss(ctx, KC_STAGE_QUANT_X);
    launch_act_records(kq_in, h, nullptr, W.meta.slot_tok, A, d, W.xrec, A, nullptr,
                       mma_gu && any_large ? W.x16 : nullptr, st, W.meta.offsets + E);
    CKL();
  }
  // 4. gate and up products -> g, u [slot, ff].
  if (fork) RC(fork_aux());
  if (any_large && mma_gu) {
    StageScope ss(ctx, KC_STAGE_GATE_UP_F32);
    const MmaMaps* tmap = nullptr;
    if (cached_tmaps(W.map_x16, W.x16, A, d, tmap) != KC_OK) return fail(ctx, KC_ERR_CUDA, "tensor map (x16) failed");
    MmaArgs ma{};
    ma.part = W.mma_part;
    ma.tile_cnt = W.mma_cnt;
    ma.w[0] = L.gate;
    ma.w[1] = L.up;
    ma.n_mat = 2;
    ma.expert_stride = L.mb_gate;
    ma.expert_base = ebase;
    ma.slot = L.slot;
    ma.rows = ff;
    ma.cols = d;
    ma.type = L.t_gate;
    ma.list = W.meta.large_list;
    ma.n_list = W.meta.n_lists + 1;
    ma.offsets = W.meta.offsets;
    ma.tt_prefix = W.meta.large_tt;
    ma.out[0] = W.g;
    ma.out[1] = W.u;
    ma.out_stride = ff;
    ma.status = ctx->status;
    ma.wide = (int64_t)A > 256LL * E;  // more than 256 rows per expert expected
    ma.bn = std::min(n_rows, kMmaTileN);  // a token adds at most one row to an expert
    ma.read_once = n_rows <= kMmaTileN;
    RC(launch_mma_grouped(ma, *tmap, max_tt * ceil_div(ff, 128), lst));
    CKL();
  } else if (any_large) {
    GroupedArgs g = grouped_base(ctx);
    g.w0 = L.gate;
    g.w1 = L.up;
    g.expert_stride = L.mb_gate;
    g.expert_base = ebase;
    g.slot = L.slot;
    g.rows = ff;
    g.cols = d;
    g.type = L.t_gate;
    g.offsets = W.meta.offsets;
    g.slot_src = W.meta.slot_tok;
    g.af = h;
    g.out = W.g;
    g.out2 = W.u;
    g.out_stride = ff;
    g.list = W.meta.large_list;
    g.n_list = W.meta.n_lists + 1;
    StageScope ss(ctx, KC_STAGE_GATE_UP_F32);
    RC(launch_grouped_f32(g, true, std::min(E, A / 4), n_rows, lst));
    CKL();
  }
  {
    StageScope ss(ctx, KC_STAGE_GATE_UP_INT8);
    DecodeArgs dg{};
    dg.w[0] = L.gate;
    dg.w[1] = L.up;
    dg.n_mat = 2;
    dg.expert_stride = L.mb_gate;
    dg.expert_base = ebase;
    dg.slot = L.slot;
    dg.rows = ff;
    dg.cols = d;
    dg.type = L.t_gate;
    dg.list = W.meta.small_list;
    dg.n_list = W.meta.n_lists;
    dg.offsets = W.meta.offsets;
    dg.n_experts = E;
    dg.early = !(dispatched && recorded);  // the list is older than the launch just before
    dg.rec = W.xrec;
    dg.rec_slots = A;
    dg.out[0] = W.g;
    dg.out[1] = W.u;
    dg.out_stride = ff;
    dg.status = ctx->status;
    RC(launch_decode(dg, max_small * 2 * ceil_div(ff, kTileRows), st, dec_ctas));
    CKL();
  }
  if (fork) RC(join_aux());
  // 5. SwiGLU of every slot -> act (f32) and its activation records.
  {
    StageScope ss(ctx, KC_STAGE_QUANT_ACT);
    launch_act_records(kq_dn, W.g, W.u, nullptr, A, ff, W.arec, A, any_large ? W.act : nullptr,
                       any_large && mma_dn ? W.act16 : nullptr, st, W.meta.offsets + E);
    CKL();
  }
  // 6. down -> y [slot, d].
  if (fork) RC(fork_aux());
  if (any_large && mma_dn) {
    StageScope ss(ctx, KC_STAGE_DOWN_F32);
    const MmaMaps* tmap = nullptr;
    if (cached_tmaps(W.map_act16, W.act16, A, ff, tmap) != KC_OK)
      return fail(ctx, KC_ERR_CUDA, "tensor map (act16) failed");
    MmaArgs ma{};
    ma.part = W.mma_part;
    ma.tile_cnt = W.mma_cnt;
    ma.w[0] = L.down;
    ma.n_mat = 1;
    ma.expert_stride = L.mb_down;
    ma.expert_base = ebase;
    ma.slot = L.slot;
    ma.rows = d;
    ma.cols = ff;
    ma.type = L.t_down;
    ma.list = W.meta.large_list;
    ma.n_list = W.meta.n_lists + 1;
    ma.offsets = W.meta.offsets;
    ma.tt_prefix = W.meta.large_tt;
    ma.out[0] = W.y;
    ma.out_stride = d;
    ma.status = ctx->status;
    ma.wide = (int64_t)A > 256LL * E;
    ma.bn = std::min(n_rows, kMmaTileN);
    ma.read_once = n_rows <= kMmaTileN;
    RC(launch_mma_grouped(ma, *tmap, max_tt * ceil_div(d, 128), lst));
    CKL();
  } else if (any_large) {
    GroupedArgs dn = grouped_base(ctx);
    dn.w0 = L.down;
    dn.expert_stride = L.mb_down;
    dn.expert_base = ebase;
    dn.slot = L.slot;
    dn.rows = d;
    dn.cols = ff;
    dn.type = L.t_down;
    dn.offsets = W.meta.offsets;
    dn.slot_src = nullptr;
    dn.af = W.act;
    dn.out = W.y;
    dn.out_stride = d;
    dn.list = W.meta.large_list;
    dn.n_list = W.meta.n_lists + 1;
    StageScope ss(ctx, KC_STAGE_DOWN_F32);
    RC(launch_grouped_f32(dn, false, std::min(E, A / 4), n_rows, lst));
    CKL();
  }
  {
    StageScope ss(ctx, KC_STAGE_DOWN_INT8);
    DecodeArgs dd{};
    dd.w[0] = L.down;
    dd.n_mat = 1;
    dd.expert_stride = L.mb_down;
    dd.expert_base = ebase;
    dd.slot = L.slot;
    dd.rows = d;
    dd.cols = ff;
    dd.type = L.t_down;
    dd.list = W.meta.small_list;
    dd.n_list = W.meta.n_lists;
    dd.offsets = W.meta.offsets;
    dd.n_experts = E;
    dd.early = true;  // the list was built before the SwiGLU records launch
    dd.rec = W.arec;
    dd.rec_slots = A;
    dd.out[0] = W.y;
    dd.out_stride = d;
    dd.status = ctx->status;
    RC(launch_decode(dd, max_small * ceil_div(d, kTileRows), st, dec_ctas));
    CKL();
  }
  if (fork) RC(join_aux());
  return KC_OK;
}

// quant::matmul of an uploaded dense matrix D on device rows x [n, cols] ->
// out [n, rows] (quant.rs:229-339 dispatch: F32 -> router kernel order, n < 4
// -> int8 decode, n >= 4 -> tcgen05, else CUDA-core f32). Uses the workspace's
// records, f16 copy and dispatch metadata, which must already hold n rows of
// D.cols values (it is grown here only if it does not).
// rec_ready (optional, K-quant D, n < 4): x's Q8_K records already made
// ([cols / 256][n] records), e.g. by the RMSNorm that produced x.
static int dense_forward(kc_ctx* ctx, const Dense& D, const float* x, int n, float* out,
                         const uint8_t* rec_ready = nullptr, int64_t out_stride = 0) {
  if (out_stride <= 0) out_stride = D.rows;
  if (n == 0) return KC_OK;
  cudaStream_t st = ctx->stream;
  if (D.t == T_F32) {
    launch_router_logits(reinterpret_cast<const float*>(D.w), D.rs / 4, (int)D.rows, (int)D.cols, x, n, out, ctx->status,
                         st, ctx->rows_mode);
    CKL();
    return KC_OK;
  }
  // By rows (n >= 4): groups of at most three rows on the int8 path, each
  // group a list entry over the same matrix.
  const bool by_rows = ctx->rows_mode && n >= 4;
  const int groups = by_rows ? (n + 2) / 3 : 1;
  RC(ensure_work(ctx, n, groups, 1, (int)std::min<int64_t>(D.cols, 1 << 30), 256));
  Work& W = ctx->ws;
  const int meta_key = by_rows ? -n : n;
  const bool meta_ready = W.dmeta_n == meta_key;
  if (!meta_ready) {
    launch_dense_meta(n, W.dmeta, st, by_rows);
    CKL();
    W.dmeta_n = meta_key;
  }
  const DispatchOut& M = W.dmeta;
  GroupedArgs a = grouped_base(ctx);
  a.w0 = D.w;
  a.expert_stride = 0;
  a.expert_base = 0;
  a.rows = (int)D.rows;
  a.cols = (int)D.cols;
  a.type = D.t;
  a.offsets = M.offsets;
  a.slot_src = nullptr;
  a.af = x;
  a.out = out;
  a.out_stride = out_stride;
  if (n < 4 || by_rows) {
    const bool kq = is_k(D.t);
    const bool ready = rec_ready && kq;
    if (!ready) {
      launch_act_records(kq, x, nullptr, nullptr, n, D.cols, W.xrec, n, nullptr, nullptr, st);
      CKL();
    }
    DecodeArgs dv{};
    dv.w[0] = D.w;
    dv.n_mat = 1;
    dv.rows = (int)D.rows;
    dv.cols = (int)D.cols;
    dv.type = D.t;
    dv.list = M.small_list;
    dv.n_list = M.n_lists;
    dv.offsets = M.offsets;
    dv.n_experts = groups;
    dv.tile_major = by_rows;
    dv.early = meta_ready;
    dv.rec = ready ? rec_ready : W.xrec;
    dv.rec_slots = n;
    dv.out[0] = out;
    dv.out_stride = out_stride;
    dv.status = ctx->status;
    RC(launch_decode(dv, groups * ceil_div(D.rows, kTileRows), st));
  } else if (!ctx->f32_prefill && mma_supported(D.t, D.cols, 1)) {
    launch_act_records(is_k(D.t), x, nullptr, nullptr, n, D.cols, nullptr, n, nullptr, W.x16, st);
    CKL();
    const MmaMaps* tmap = nullptr;
    if (cached_tmaps(W.map_x16, W.x16, n, D.cols, tmap) != KC_OK)
      return fail(ctx, KC_ERR_CUDA, "tensor map (x16) failed");
    MmaArgs ma{};
    ma.part = W.mma_part;
    ma.tile_cnt = W.mma_cnt;
    ma.w[0] = D.w;
    ma.n_mat = 1;
    ma.rows = (int)D.rows;
    ma.cols = (int)D.cols;
    ma.type = D.t;
    ma.list = M.large_list;
    ma.n_list = M.n_lists + 1;
    ma.offsets = M.offsets;
    ma.tt_prefix = M.large_tt;
    ma.out[0] = out;
    ma.out_stride = out_stride;
    ma.status = ctx->status;
    ma.wide = n > 256;
    ma.bn = std::min(n, kMmaTileN);
    ma.read_once = n <= kMmaTileN;
    RC(launch_mma_grouped(ma, *tmap, ceil_div(n, kMmaTileN) * ceil_div(D.rows, 128), st));
  } else {
    a.list = M.large_list;
    a.n_list = M.n_lists + 1;
    RC(launch_grouped_f32(a, false, 1, n, st));
  }
  CKL();
  return KC_OK;
}

static Dense as_dense(const Layer::Mat& m) {
  Dense D;
  D.t = m.t;
  D.rows = m.rows;
  D.cols = m.cols;
  D.rs = round16(m.cols * 4);
  D.w = m.w;
  return D;
}

// Workspace columns the layer's products need (routed experts and shared
// expert): D >= d and the shared ff, F >= ff and the shared ff.
static int layer_work_d(const Layer& L) { return std::max(L.d, L.has_shared ? L.sh_ff : 0); }
static int layer_work_f(const Layer& L) { return std::max(L.ff, L.has_shared ? L.sh_ff : 0); }

// The shared expert's contribution (transformer.rs:571-587): g = gate h,
// u = up h, g = g / (1 + exp(-g)) * u, y = down g, then
// out[s] += sigmoid(gate_inp . h[s]) * y[s] (gate 1 without gate_inp). The
// matmuls follow quant::matmul's dispatch on the token count, like
// Transformer::mm. Runs after the routed experts' combine.
static int shared_forward(kc_ctx* ctx, const Layer& L, const float* h, int n_tok, float* out) {
  if (!L.has_shared || n_tok == 0) return KC_OK;
  Work& W = ctx->ws;
  cudaStream_t st = ctx->stream;
  const int d = L.d, sf = L.sh_ff;
  RC(dense_forward(ctx, as_dense(L.sh_gate), h, n_tok, W.g));
  RC(dense_forward(ctx, as_dense(L.sh_up), h, n_tok, W.u));
  launch_act_records(false, W.g, W.u, nullptr, n_tok, sf, nullptr, n_tok, W.act, nullptr, st);
  CKL();
  RC(dense_forward(ctx, as_dense(L.sh_down), W.act, n_tok, W.y));
  if (L.sh_inp) {
    launch_router_logits(L.sh_inp, d, 1, d, h, n_tok, W.logits, ctx->status, st, /*force_dot=*/true);
    CKL();
  }
  launch_shared_add(W.y, L.sh_inp ? W.logits : nullptr, n_tok, d, out, st);
  CKL();
  return KC_OK;
}

// ---- expert parallelism --------------------------------------------------
template <typename P>
static int regrow(P*& p, size_t bytes) {
  if (p) cudaFree(p);
  p = nullptr;
  return cudaMalloc(reinterpret_cast<void**>(&p), std::max<size_t>(bytes, 256)) == cudaSuccess ? KC_OK : KC_ERR_OOM;
}

static int ep_grow_home(kc_ctx* ctx, int T, int k, int d) {
  EpBufs& B = ctx->epb;
  const int G = ctx->ep.world;
  if (T <= B.T && k <= B.k && d <= B.d && B.ids_home) return KC_OK;
  CK(cudaStreamSynchronize(ctx->stream));
  T = std::max(T, B.T);
  k = std::max(k, B.k);
  d = std::max(d, B.d);
  const size_t tk = (size_t)T * k;
  int rc = KC_OK;
  if (rc == KC_OK) rc = regrow(B.ids_home, tk * 4);
  if (rc == KC_OK) rc = regrow(B.w_home, tk * 4);
  if (rc == KC_OK) rc = regrow(B.send_tok, (size_t)G * T * 4);
  if (rc == KC_OK) rc = regrow(B.ret_pos, tk * 4);
  if (rc == KC_OK) rc = regrow(B.xch, (size_t)4 * kEpMaxWorld * 4);
  if (rc == KC_OK) rc = regrow(B.sendbuf, (size_t)G * T * d * 4);
  if (rc == KC_OK) rc = regrow(B.sendmeta, (size_t)G * T * 2 * k * 4);
  if (rc == KC_OK) rc = regrow(B.retrecv, tk * d * 4);
  if (rc == KC_OK && !B.xch_host && cudaMallocHost(reinterpret_cast<void**>(&B.xch_host), 4 * kEpMaxWorld * 4) != cudaSuccess)
    rc = KC_ERR_OOM;
  if (rc != KC_OK) return fail(ctx, rc, "expert-parallel buffers: device allocation failed");
  B.T = T;
  B.k = k;
  B.d = d;
  return KC_OK;
}

static int ep_grow_owner(kc_ctx* ctx, int R, int RS, int k, int d) {
  EpBufs& B = ctx->epb;
  if (R <= B.R && RS <= B.RS && k <= B.k && d <= B.d && B.recvbuf) return KC_OK;
  CK(cudaStreamSynchronize(ctx->stream));
  R = std::max(std::max(R, B.R), 1);
  RS = std::max(std::max(RS, B.RS), 1);
  const size_t rk = (size_t)R * k;
  int rc = KC_OK;
  if (rc == KC_OK) rc = regrow(B.recvbuf, (size_t)R * d * 4);
  if (rc == KC_OK) rc = regrow(B.recvmeta, rk * 2 * 4);
  if (rc == KC_OK) rc = regrow(B.ids_loc, rk * 4);
  if (rc == KC_OK) rc = regrow(B.w_loc, rk * 4);
  if (rc == KC_OK) rc = regrow(B.ret_send_pos, rk * 4);
  if (rc == KC_OK) rc = regrow(B.retsend, (size_t)RS * d * 4);
  if (rc != KC_OK) return fail(ctx, rc, "expert-parallel buffers: device allocation failed");
  B.R = R;
  B.RS = RS;
  return KC_OK;
}

static void ep_free_bufs(EpBufs& B) {
  void* ps[] = {B.ids_home, B.w_home, B.send_tok, B.ret_pos, B.xch, B.sendbuf, B.sendmeta, B.retrecv,
                B.recvbuf, B.recvmeta, B.ids_loc, B.w_loc, B.ret_send_pos, B.retsend};
  for (void* p : ps)
    if (p) cudaFree(p);
  if (B.xch_host) cudaFreeHost(B.xch_host);
  B = EpBufs{};
}

static int ep_rc(kc_ctx* ctx, int rc) {
  return rc == KC_OK ? KC_OK : fail(ctx, rc, "expert parallel: %s", ep_last_error(ctx->ep));
}

// The expert-parallel layer on decode-sized batches (n_tok within the
// capacity mapped by kc_ep_reserve): the same steps as ep_pipeline, with every
// exchange done by this library's kernels over NVLink peer memory -- rows and
// their selections are stored straight into the owners' arenas, results
// straight into the home ranks' arenas, each followed by a published sequence
// number that the receiver waits for on the device. No host synchronisation,
// no NCCL call. The owner runs its experts on the arena's fixed-capacity
// layout ([source][capacity] rows; rows beyond a source's count carry no
// selection).
static int ep_pipeline_p2p(kc_ctx* ctx, const Layer& L, const float* router, const float* h, int n_tok,
                           float* out, int32_t* ids_out, float* w_out) {
  EpState& S = ctx->ep;
  const int G = S.world, E = L.n_expert, k = L.k, d = L.d, ff = L.ff;
  const int epr = E / G, T = std::max(n_tok, 1);
  EpBufs& B = ctx->epb;
  cudaStream_t st = ctx->stream;
  if (n_tok > 0) {
    {
      StageScope ss(ctx, KC_STAGE_ROUTER_LOGITS);
      launch_router_logits(router, d, E, d, h, n_tok, ctx->ws.logits, ctx->status, st, ctx->rows_mode);
      CKL();
    }
    StageScope ss(ctx, KC_STAGE_ROUTE);
    launch_route(ctx->ws.logits, n_tok, E, k, L.norm_topk, L.weights_scale, B.ids_home, B.w_home, st);
    CKL();
  }
  const int R = G * S.p2p.T;  // owner-side rows: every source's capacity
  RC(ep_grow_owner(ctx, R, 1, k, d));
  Work& WO = ctx->ws_ep;
  RC(ensure_work(ctx, WO, R, epr, k, d, ff));
  // Every host-side step that can fail comes before the sequence number
  // moves on, so that the ranks' sequence numbers stay equal.
  ++S.p2p.seq;
  const EpP2PArgs pa = ep_p2p_args(S, ctx->status);
  {
    StageScope ss(ctx, KC_STAGE_DISPATCH);
    launch_ep_plan(B.ids_home, n_tok, k, G, epr, T, B.send_tok, B.ret_pos, B.xch, st, S.p2p.ret_cap);
    launch_ep_p2p_send(pa, h, B.ids_home, B.w_home, B.send_tok, B.xch, T, st);
    launch_ep_p2p_wait(pa, 0, st);
    launch_ep_p2p_local_ids(pa, L.first_expert, epr, B.ids_loc, B.w_loc, st);
    CKL();
  }
  Layer LL = L;
  LL.n_expert = epr;
  RC(experts_forward(ctx, WO, LL, epr, 0, reinterpret_cast<const float*>(S.p2p.arena), R, B.ids_loc, B.w_loc, k));
  launch_ep_p2p_ret_plan(B.ids_loc, G, S.p2p.T, k, B.ret_send_pos, st);
  launch_ep_p2p_ret_send(pa, WO.y, WO.meta.tok_slot, B.ret_send_pos, st);
  launch_ep_p2p_wait(pa, 1, st);
  CKL();
  if (n_tok > 0) {
    StageScope ss(ctx, KC_STAGE_COMBINE);
    launch_combine(reinterpret_cast<const float*>(S.p2p.arena + S.p2p.off_ret), B.ret_pos, B.ids_home, B.w_home,
                   n_tok, k, d, out, st);
    CKL();
  }
  if (ids_out && n_tok > 0)
    CK(cudaMemcpyAsync(ids_out, B.ids_home, (size_t)n_tok * k * 4, cudaMemcpyDeviceToDevice, st));
  if (w_out && n_tok > 0)
    CK(cudaMemcpyAsync(w_out, B.w_home, (size_t)n_tok * k * 4, cudaMemcpyDeviceToDevice, st));
  RC(shared_forward(ctx, L, h, n_tok, out));
  return KC_OK;
}

// Transformer::moe_ffn with the experts sharded over the group: route this
// rank's tokens, send each token once to every rank owning one of its
// experts, run the local experts on the rows received from all ranks, send
// each (token, expert) result row back, and combine in ascending expert id.
// Every rank must make the same sequence of calls (collectives).
static int ep_pipeline(kc_ctx* ctx, const Layer& L, const float* router, const float* h, int n_tok, float* out,
                       int32_t* ids_out, float* w_out) {
  EpState& S = ctx->ep;
  const int G = S.world, me = S.rank;
  const int E = L.n_expert, k = L.k, d = L.d, ff = L.ff;
  if (E % G != 0 || L.n_local != E / G || L.first_expert != me * (E / G))
    return fail(ctx, KC_ERR_STATE, "expert parallel: layer must hold experts [%d, %d) of %d on rank %d",
                me * (E / std::max(G, 1)), (me + 1) * (E / std::max(G, 1)), E, me);
  if (d % 4) return fail(ctx, KC_ERR_SHAPE, "expert parallel: d %% 4 != 0");
  const int epr = E / G;
  const int T = std::max(n_tok, 1);
  RC(ensure_work(ctx, T, E, k, layer_work_d(L), layer_work_f(L)));
  RC(ep_grow_home(ctx, T, k, d));
  EpBufs& B = ctx->epb;
  cudaStream_t st = ctx->stream;
  if (S.p2p.ready && n_tok <= S.p2p.T && d == S.p2p.d && k == S.p2p.k)
    return ep_pipeline_p2p(ctx, L, router, h, n_tok, out, ids_out, w_out);
  if (S.p2p.ready) {
    // The peer arenas are mapped, so another rank may have taken the peer
    // path in this call (its tokens within the reserved capacity while this
    // rank's are not). An NCCL call would then wait for a rank that never
    // makes it. So announce this rank's path on every rank's line, wait for
    // every rank's announcement (bounded) and compare, and make no NCCL call
    // unless all ranks took NCCL; otherwise the call fails with KC_ERR_STATE
    // on every rank (the peer-path ranks stop waiting when they see it).
    ++S.p2p.seq;
    EpP2PArgs pa = ep_p2p_args(S, ctx->status);
    pa.path = kEpPathNccl;
    launch_ep_p2p_announce(pa, st);
    launch_ep_p2p_wait(pa, 0, st);
    CKL();
    RC(check_status(ctx));
  }
  // 1. route this rank's tokens.
  if (n_tok > 0) {
    {
      StageScope ss(ctx, KC_STAGE_ROUTER_LOGITS);
      launch_router_logits(router, d, E, d, h, n_tok, ctx->ws.logits, ctx->status, st, ctx->rows_mode);
      CKL();
    }
    StageScope ss(ctx, KC_STAGE_ROUTE);
    launch_route(ctx->ws.logits, n_tok, E, k, L.norm_topk, L.weights_scale, B.ids_home, B.w_home, st);
    CKL();
  }
  // 2. plan and pack the rows for every owner; exchange the counts.
  int* xch_out = B.xch;
  int* xch_in = B.xch + 2 * kEpMaxWorld;
  {
    StageScope ss(ctx, KC_STAGE_DISPATCH);
    launch_ep_plan(B.ids_home, n_tok, k, G, epr, T, B.send_tok, B.ret_pos, xch_out, st);
    launch_ep_pack(h, B.ids_home, B.w_home, B.send_tok, xch_out, G, T, k, d, B.sendbuf, B.sendmeta, st);
    CKL();
    RC(ep_rc(ctx, ep_exchange_counts(S, xch_out, xch_in, st)));
    CK(cudaMemcpyAsync(B.xch_host, B.xch, 4 * kEpMaxWorld * sizeof(int), cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
  }
  const int* ho = B.xch_host;                   // [r]: rows sent to r, result rows expected from r
  const int* hi = B.xch_host + 2 * kEpMaxWorld;  // [r]: rows received from r, result rows owed to r
  int64_t so[kEpMaxWorld], sb[kEpMaxWorld], ro[kEpMaxWorld], rb[kEpMaxWorld];
  int64_t mso[kEpMaxWorld], msb[kEpMaxWorld], mro[kEpMaxWorld], mrb[kEpMaxWorld];
  int64_t yso[kEpMaxWorld], ysb[kEpMaxWorld], yro[kEpMaxWorld], yrb[kEpMaxWorld];
  int64_t n_recv = 0, n_send = 0, n_ret_send = 0, n_ret_recv = 0;
  for (int q = 0; q < G; ++q) {
    so[q] = n_send * d * 4;
    sb[q] = (int64_t)ho[2 * q] * d * 4;
    mso[q] = n_send * 2 * k * 4;
    msb[q] = (int64_t)ho[2 * q] * 2 * k * 4;
    ro[q] = n_recv * d * 4;
    rb[q] = (int64_t)hi[2 * q] * d * 4;
    mro[q] = n_recv * 2 * k * 4;
    mrb[q] = (int64_t)hi[2 * q] * 2 * k * 4;
    yso[q] = n_ret_send * d * 4;
    ysb[q] = (int64_t)hi[2 * q + 1] * d * 4;
    yro[q] = n_ret_recv * d * 4;
    yrb[q] = (int64_t)ho[2 * q + 1] * d * 4;
    n_send += ho[2 * q];
    n_recv += hi[2 * q];
    n_ret_send += hi[2 * q + 1];
    n_ret_recv += ho[2 * q + 1];
  }
  if (n_ret_recv != (int64_t)n_tok * k || n_recv > (int64_t)1 << 30)
    return fail(ctx, KC_ERR_STATE, "expert parallel: inconsistent exchange counts");
  RC(ep_grow_owner(ctx, (int)n_recv, (int)n_ret_send, k, d));
  // 3. rows and their selections to the owners.
  {
    const EpA2A parts[2] = {{B.sendbuf, so, sb, B.recvbuf, ro, rb}, {B.sendmeta, mso, msb, B.recvmeta, mro, mrb}};
    RC(ep_rc(ctx, ep_alltoallv(S, parts, 2, st)));
  }
  // 4. the local experts on every received row.
  if (n_recv > 0) {
    const int nr = (int)n_recv;
    launch_ep_local_ids(B.recvmeta, nr, k, L.first_expert, epr, B.ids_loc, B.w_loc, st);
    CKL();
    Work& WO = ctx->ws_ep;
    RC(ensure_work(ctx, WO, nr, epr, k, d, ff));
    Layer LL = L;
    LL.n_expert = epr;
    RC(experts_forward(ctx, WO, LL, epr, 0, B.recvbuf, nr, B.ids_loc, B.w_loc, k));
    launch_ep_ret_plan(B.ids_loc, nr, k, B.ret_send_pos, st);
    launch_ep_ret_pack(WO.y, WO.meta.tok_slot, B.ret_send_pos, nr, k, d, (int)n_ret_send, B.retsend, st);
    CKL();
  }
  // 5. result rows back to their tokens' ranks; combine in ascending expert id.
  {
    const EpA2A parts[1] = {{B.retsend, yso, ysb, B.retrecv, yro, yrb}};
    RC(ep_rc(ctx, ep_alltoallv(S, parts, 1, st)));
  }
  if (n_tok > 0) {
    StageScope ss(ctx, KC_STAGE_COMBINE);
    launch_combine(B.retrecv, B.ret_pos, B.ids_home, B.w_home, n_tok, k, d, out, st);
    CKL();
  }
  if (ids_out && n_tok > 0)
    CK(cudaMemcpyAsync(ids_out, B.ids_home, (size_t)n_tok * k * 4, cudaMemcpyDeviceToDevice, st));
  if (w_out && n_tok > 0)
    CK(cudaMemcpyAsync(w_out, B.w_home, (size_t)n_tok * k * 4, cudaMemcpyDeviceToDevice, st));
  // The shared expert is dense and replicated: every rank adds it for its own tokens.
  RC(shared_forward(ctx, L, h, n_tok, out));
  return KC_OK;
}

// defer_combine (one GPU, no shared expert): the combine may be left to the
// caller (the model's next RMSNorm), which then reads W.y, W.meta.tok_slot,
// W.ids and W.w before anything else touches the workspace, and out is not
// written; *deferred says whether it was.
static int moe_pipeline(kc_ctx* ctx, const Layer& L, const float* router, const float* h, int n_tok, float* out,
                        int32_t* ids_out, float* w_out, bool defer_combine = false, bool* deferred = nullptr) {
  if (deferred) *deferred = false;
  if (L.streamed && ctx->ep.world > 1)
    return fail(ctx, KC_ERR_STATE, "layer %d: host-streamed experts are not served by expert parallelism", L.id);
  if (ctx->ep.world > 1) return ep_pipeline(ctx, L, router, h, n_tok, out, ids_out, w_out);
  const int E = L.n_expert, k = L.k, d = L.d;
  RC(ensure_work(ctx, n_tok, E, k, layer_work_d(L), layer_work_f(L)));
  Work& W = ctx->ws;
  cudaStream_t st = ctx->stream;
  if (n_tok == 0) return KC_OK;
  // 1. router logits and top-k (Transformer::route).
  {
    StageScope ss(ctx, KC_STAGE_ROUTER_LOGITS);
    launch_router_logits(router, d, E, d, h, n_tok, W.logits, ctx->status, st, ctx->rows_mode);
    CKL();
  }
  // Small batches: route and dispatch in one launch, for decode batches with
  // the input records too.
  const bool with_rec = is_k(L.t_gate) && route_dispatch_supported(n_tok, E, k, d, true);
  const bool front = !ctx->prof.on && (with_rec || route_dispatch_supported(n_tok, E, k, d, false));
  if (front) {
    launch_route_dispatch(W.logits, n_tok, E, k, L.norm_topk, L.weights_scale, W.ids, W.w, W.meta, h, d,
                          with_rec ? W.xrec : nullptr, st, ctx->rows_mode);
    CKL();
  } else {
    StageScope ss(ctx, KC_STAGE_ROUTE);
    launch_route(W.logits, n_tok, E, k, L.norm_topk, L.weights_scale, W.ids, W.w, st);
    CKL();
  }
  // Host-streamed experts: the routed ones copied into HBM slots.
  Layer Ls;
  const Layer* LE = &L;
  if (L.streamed) {
    StageScope ss(ctx, KC_STAGE_EXPERT_LOAD);
    RC(streams_demand(ctx, L, W.ids, n_tok * k, Ls));
    LE = &Ls;
  }
  // 2-6. dispatch, records, gate/up, SwiGLU, down.
  RC(experts_forward(ctx, W, *LE, E, LE->first_expert, h, n_tok, W.ids, W.w, k, front, front && with_rec));
  // 7. combine (un-permute, ascending expert id).
  if (!defer_combine || L.has_shared) {
    StageScope ss(ctx, KC_STAGE_COMBINE);
    launch_combine(W.y, W.meta.tok_slot, W.ids, W.w, n_tok, k, d, out, st);
    CKL();
  } else if (deferred) {
    *deferred = true;
  }
  if (ids_out) CK(cudaMemcpyAsync(ids_out, W.ids, (size_t)n_tok * k * 4, cudaMemcpyDeviceToDevice, st));
  if (w_out) CK(cudaMemcpyAsync(w_out, W.w, (size_t)n_tok * k * 4, cudaMemcpyDeviceToDevice, st));
  // 8. shared expert (qwen2moe), after the routed experts.
  RC(shared_forward(ctx, L, h, n_tok, out));
  return KC_OK;
}

// ===========================================================================
// The dense decode path of a whole model (Transformer::forward,
// transformer.rs:287-302, 375-467): embedding rows, per layer RMSNorm ->
// q/k/v -> bias / q-k norm / RoPE -> f16 KV cache -> causal GQA attention ->
// output projection -> residual -> RMSNorm -> FFN (routed experts through
// moe_pipeline, or dense SwiGLU) -> residual; then the final norm, the output
// head and argmax. The matvecs go through dense_forward (quant::matmul's
// dispatch), so decode steps run the int8 path bit for bit.
constexpr int kModelBatch = 256;  // Transformer::n_batch (transformer.rs:269)
constexpr int kMaxSequences = 32;  // rows of a batch step (route_dispatch's one token mask word per expert)

struct Model {
  int n_layer = 0, d = 0, nh = 0, nkv = 0, hd = 0, n_vocab = 0, n_ctx = 0, rd = 0, arch = 0;
  float eps = 0.f, rope_base = 0.f;
  struct Lay {
    float *attn_norm = nullptr, *ffn_norm = nullptr, *qn = nullptr, *kn = nullptr;
    float *bq = nullptr, *bk = nullptr, *bv = nullptr;
    Dense q, k, v, o, qkv, gate, up, down;
  };
  std::vector<Lay> L;
  uint8_t* embd = nullptr;  // raw GGUF rows (get_row)
  int embd_t = -1;
  int64_t embd_rb = 0;
  float* out_norm = nullptr;
  Dense output;
  bool ready = false;
  // KV caches of n_seq sequences, [n_seq][n_layer][n_ctx][nkv * hd] each;
  // the single-sequence calls (kc_model_forward / _generate) use sequence 0.
  __half* kc = nullptr;
  __half* vc = nullptr;
  int n_seq = 1;
  float2* rope = nullptr;  // [n_ctx][rd / 2] (sin, cos)
  int cached = 0;
  int cur = 0;  // sequence whose cache the single-sequence path uses
  int* row_pos = nullptr;    // [n_seq] positions of the rows of a batch step
  uint32_t* seq_tok = nullptr;  // [n_seq] each sequence's pending token (kc_model_prefill_seq / _decode_seqs)
  std::vector<int> seq_pos;     // positions each sequence holds (-1: none yet); [0] mirrors `cached`
  int64_t seq_elems() const { return (int64_t)n_layer * n_ctx * nkv * hd; }
  // Activations for up to T tokens per forward chunk.
  int T = 0, F = 0;
  float *x = nullptr, *h = nullptr, *qkv = nullptr, *q = nullptr, *att = nullptr, *tmp = nullptr, *ffn = nullptr;
  float *g = nullptr, *u = nullptr, *logits = nullptr;
  uint32_t* tok = nullptr;  // [T]
  uint8_t* rec = nullptr;   // Q8_K records of the attention norm's output (decode steps)
  uint32_t* next = nullptr; // argmax result ([n_seq] in a batch step)
  int* counters = nullptr;  // [0] generated-token index, [1] position (graph-replayed decode steps)
  // Router lookahead of host-streamed layers: the next layer's norm of up to
  // 4 rows, its logits, ids and weights.
  float* look = nullptr;
  int64_t bytes = 0;
};

void free_layer(Layer& L) {
  if (L.host) cudaFreeHost(L.host);
  cudaFree(L.gate);
  cudaFree(L.up);
  cudaFree(L.down);
  cudaFree(L.router);
  cudaFree(L.sh_gate.w);
  cudaFree(L.sh_up.w);
  cudaFree(L.sh_down.w);
  cudaFree(L.sh_inp);
  L = Layer{};
}

void free_dense(kc_ctx* ctx, Dense& D) {
  if (D.w) cudaFree(D.w);
  D = Dense{};
  (void)ctx;
}

void model_free(kc_ctx* ctx) {
  Model* m = ctx->model;
  if (!m) return;
  for (auto& l : m->L) {
    for (float* v : {l.attn_norm, l.ffn_norm, l.qn, l.kn, l.bq, l.bk, l.bv}) cudaFree(v);
    for (Dense* D : {&l.q, &l.k, &l.v, &l.o, &l.qkv, &l.gate, &l.up, &l.down}) free_dense(ctx, *D);
  }
  cudaFree(m->embd);
  cudaFree(m->out_norm);
  free_dense(ctx, m->output);
  cudaFree(m->kc);
  cudaFree(m->vc);
  cudaFree(m->rope);
  for (void* p : {(void*)m->x, (void*)m->h, (void*)m->qkv, (void*)m->q, (void*)m->att, (void*)m->tmp,
                  (void*)m->ffn, (void*)m->g, (void*)m->u, (void*)m->logits, (void*)m->tok, (void*)m->next,
                  (void*)m->counters, (void*)m->rec, (void*)m->row_pos, (void*)m->seq_tok, (void*)m->look})
    cudaFree(p);
  delete m;
  ctx->model = nullptr;
}

int model_dense(kc_ctx* ctx, Dense& D, int t, const void* w, int64_t rows, int64_t cols, bool on_dev) {
  free_dense(ctx, D);
  D.t = t;
  D.rows = rows;
  D.cols = cols;
  D.rs = round16(cols * 4);
  CK(cudaMalloc(&D.w, dev_matrix_bytes(t, rows, cols)));
  RC(upload_matrix(ctx, t, w, 1, rows, cols, D.w, on_dev));
  return KC_OK;
}

int model_vec(kc_ctx* ctx, float*& dst, const void* w, int64_t n, bool on_dev) {
  cudaFree(dst);
  dst = nullptr;
  CK(cudaMalloc(&dst, n * 4));
  CK(cudaMemcpyAsync(dst, w, n * 4, on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->stream));
  return KC_OK;
}

// Activation buffers for T tokens.
int model_buffers(kc_ctx* ctx, Model& m, int T) {
  int F = 256;
  for (auto& l : m.L)
    if (l.gate.w) F = std::max<int>(F, (int)l.gate.rows);
  if (T <= m.T && F <= m.F) return KC_OK;
  T = std::max(T, m.T);
  CK(cudaStreamSynchronize(ctx->stream));
  for (void* p : {(void*)m.x, (void*)m.h, (void*)m.qkv, (void*)m.q, (void*)m.att, (void*)m.tmp, (void*)m.ffn,
                  (void*)m.g, (void*)m.u, (void*)m.tok, (void*)m.rec})
    cudaFree(p);
  const int width = (m.nh + 2 * m.nkv) * m.hd;
  CK(cudaMalloc(&m.x, (size_t)T * m.d * 4));
  CK(cudaMalloc(&m.h, (size_t)T * m.d * 4));
  CK(cudaMalloc(&m.qkv, (size_t)T * width * 4));
  CK(cudaMalloc(&m.q, (size_t)T * m.nh * m.hd * 4));
  CK(cudaMalloc(&m.att, (size_t)T * m.nh * m.hd * 4));
  CK(cudaMalloc(&m.tmp, (size_t)T * m.d * 4));
  CK(cudaMalloc(&m.ffn, (size_t)T * m.d * 4));
  CK(cudaMalloc(&m.g, (size_t)T * F * 4));
  CK(cudaMalloc(&m.u, (size_t)T * F * 4));
  CK(cudaMalloc(&m.tok, (size_t)T * 4));
  CK(cudaMalloc(&m.rec, (size_t)std::max(std::min(T, 3), m.n_seq) * rec_row_bytes(true, std::max(256, m.d))));
  m.T = T;
  m.F = F;
  return KC_OK;
}

// First forward: check the tensors, fuse q/k/v into one matrix where their
// types and row lengths agree (each row's arithmetic is unchanged), tie the
// output head to the embedding if there is no output tensor.
int model_finalize(kc_ctx* ctx, Model& m) {
  if (m.ready) return KC_OK;
  if (!m.embd || !m.out_norm) return fail(ctx, KC_ERR_STATE, "kc_model_forward: embedding or output norm missing");
  if (!m.output.w) {
    RC(model_dense(ctx, m.output, m.embd_t, m.embd, m.n_vocab, m.d, true));
  }
  for (int l = 0; l < m.n_layer; ++l) {
    Model::Lay& y = m.L[l];
    if (!y.attn_norm || !y.ffn_norm || !y.q.w || !y.k.w || !y.v.w || !y.o.w)
      return fail(ctx, KC_ERR_STATE, "kc_model_forward: layer %d lacks an attention tensor or a norm", l);
    // A layer with dense FFN tensors is dense; otherwise it needs routed experts.
    const bool dense = y.gate.w || y.up.w || y.down.w;
    const bool moe = !dense && ctx->layers.count(l) && ctx->layers[l].has_experts && ctx->layers[l].has_router;
    if (dense && !(y.gate.w && y.up.w && y.down.w))
      return fail(ctx, KC_ERR_STATE, "kc_model_forward: layer %d lacks a dense FFN tensor", l);
    if (!dense && !moe)
      return fail(ctx, KC_ERR_STATE, "kc_model_forward: layer %d has neither routed experts nor a dense FFN", l);
    if (moe && ctx->layers[l].d != m.d) return fail(ctx, KC_ERR_SHAPE, "kc_model_forward: layer %d expert d", l);
    if (moe && ctx->ep.world <= 1 && ctx->layers[l].n_local != ctx->layers[l].n_expert)
      return fail(ctx, KC_ERR_STATE, "kc_model_forward: layer %d holds an expert shard outside an expert-parallel "
                                     "group", l);
    if (dense && (y.gate.cols != m.d || y.up.rows != y.gate.rows || y.down.rows != m.d || y.down.cols != y.gate.rows))
      return fail(ctx, KC_ERR_SHAPE, "kc_model_forward: layer %d dense FFN shapes", l);
    if (y.q.rows != (int64_t)m.nh * m.hd || y.k.rows != (int64_t)m.nkv * m.hd || y.v.rows != (int64_t)m.nkv * m.hd ||
        y.q.cols != m.d || y.o.rows != m.d || y.o.cols != (int64_t)m.nh * m.hd)
      return fail(ctx, KC_ERR_SHAPE, "kc_model_forward: layer %d attention shapes", l);
    const bool fuse = y.q.t == y.k.t && y.q.t == y.v.t && y.k.cols == y.q.cols && y.v.cols == y.q.cols &&
                      (y.q.t == T_F32 || (y.q.rows % kTileRows == 0 && y.k.rows % kTileRows == 0));
    if (!fuse) return fail(ctx, KC_ERR_SHAPE, "kc_model_forward: layer %d q/k/v differ in type or shape", l);
    free_dense(ctx, y.qkv);
    y.qkv.t = y.q.t;
    y.qkv.rows = y.q.rows + y.k.rows + y.v.rows;
    y.qkv.cols = y.q.cols;
    y.qkv.rs = y.q.rs;
    const int64_t bq = dev_matrix_bytes(y.q.t, y.q.rows, y.q.cols), bk = dev_matrix_bytes(y.k.t, y.k.rows, y.k.cols);
    CK(cudaMalloc(&y.qkv.w, dev_matrix_bytes(y.qkv.t, y.qkv.rows, y.qkv.cols)));
    CK(cudaMemcpyAsync(y.qkv.w, y.q.w, bq, cudaMemcpyDeviceToDevice, ctx->stream));
    CK(cudaMemcpyAsync(y.qkv.w + bq, y.k.w, bk, cudaMemcpyDeviceToDevice, ctx->stream));
    CK(cudaMemcpyAsync(y.qkv.w + bq + bk, y.v.w, bk, cudaMemcpyDeviceToDevice, ctx->stream));
  }
  CK(cudaStreamSynchronize(ctx->stream));
  m.ready = true;
  return KC_OK;
}

// One forward chunk of n tokens read from `tok` (device); logits of the last
// token in m.logits and its argmax in m.next. With dev_pos the chunk's
// position is m.counters[1] on the device (a graph-replayed decode step), and
// the caller advances m.cached. rows (a batch step, ctx->rows_mode): row s is
// the next token of sequence s, at position m.row_pos[s] of its own cache;
// every row gets its logits (m.logits [n][n_vocab]) and argmax (m.next[s]).
// Transformer::lookahead_prefetch (transformer.rs:498-508) for layer l + 1
// after layer l's attention: RMSNorm of the residual with l + 1's FFN norm,
// its router and top-k, then ExpertStore::prefetch of the predicted experts.
// The three kernels run on the auxiliary stream beside layer l's routing.
// Their ids are read back at layer l's own demand synchronisation when l is
// host-streamed, else here; either way the auxiliary stream is drained
// before the residual is next written (the following layer's first norm).
int model_lookahead(kc_ctx* ctx, Model& m, int l, int n) {
  auto it = ctx->layers.find(l + 1);
  if (it == ctx->layers.end() || !it->second.streamed || !it->second.has_router || m.L[l + 1].gate.w) return KC_OK;
  const Layer& R = it->second;
  if (R.d != m.d) return KC_OK;
  cudaStream_t st = ctx->stream;
  const int E = R.n_expert, k = R.k;
  if (!m.look) CK(cudaMalloc(&m.look, (size_t)4 * (m.d + 1024 + 2 * 64) * 4));
  RC(ensure_aux(ctx));
  CK(cudaEventRecord(ctx->ev_fork, st));
  CK(cudaStreamWaitEvent(ctx->aux, ctx->ev_fork, 0));
  st = ctx->aux;
  float* look_h = m.look;
  float* logits = look_h + 4 * m.d;
  int32_t* ids = reinterpret_cast<int32_t*>(logits + 4 * 1024);
  float* w = logits + 4 * 1024 + 4 * 64;
  NormArgs na{};
  na.x = m.x;
  na.w = m.L[l + 1].ffn_norm;
  na.dim = m.d;
  na.eps = m.eps;
  na.out = look_h;
  na.rec_slots = n;
  launch_add_rmsnorm(na, n, st);
  CKL();
  launch_router_logits(R.router, R.d, E, R.d, look_h, n, logits, ctx->status, st, ctx->rows_mode);
  CKL();
  launch_route(logits, n, E, k, R.norm_topk, R.weights_scale, ids, w, st);
  CKL();
  ExpertStreams& S = ctx->xs;
  S.look_layer = l + 1;
  S.look_ids = ids;
  S.look_n = n * k;
  auto cur = ctx->layers.find(l);
  const bool cur_streamed = cur != ctx->layers.end() && cur->second.streamed && !m.L[l].gate.w;
  if (!cur_streamed) RC(streams_lookahead_now(ctx));
  return KC_OK;
}

int model_chunk(kc_ctx* ctx, Model& m, int n, const uint32_t* tok, bool dev_pos, bool rows = false) {
  cudaStream_t st = ctx->stream;
  const int d = m.d, pos0 = m.cached;
  const int* pos_dev = dev_pos ? m.counters + 1 : nullptr;
  __half* kc0 = m.kc + (rows ? 0 : (int64_t)m.cur * m.seq_elems());
  __half* vc0 = m.vc + (rows ? 0 : (int64_t)m.cur * m.seq_elems());
  const float scale = 1.0f / std::sqrt((float)m.hd);  // transformer.rs:598
  launch_embed(m.embd, m.embd_t, m.embd_rb, tok, n, d, m.n_vocab, m.x, ctx->status, st);
  CKL();
  // The previous FFN's output is added to the residual by the next norm: a
  // plain buffer, or (routed layers on one GPU without a shared expert) the
  // MoE combine itself, read from the workspace (moe_pipeline's
  // defer_combine).
  const float* resid = nullptr;
  bool pending_combine = false;
  int pending_k = 0;
  auto norm = [&](float* x, const float* w, int rows, int tok0, float* out, uint8_t* rec) {
    NormArgs na{};
    na.x = x;
    na.w = w;
    na.dim = d;
    na.eps = m.eps;
    na.out = out;
    na.rec = rec;
    na.rec_slots = rows;
    na.tok0 = tok0;
    if (pending_combine) {
      const Work& W = ctx->ws;
      na.cy = W.y;
      na.tok_slot = W.meta.tok_slot;
      na.ids = W.ids;
      na.cw = W.w;
      na.k = pending_k;
    } else if (resid) {
      na.y = resid + (int64_t)tok0 * d;
    }
    launch_add_rmsnorm(na, rows, st);
  };
  for (int l = 0; l < m.n_layer; ++l) {
    Model::Lay& y = m.L[l];
    // Decode rows with a K-quant q/k/v take their Q8_K records from the norm.
    uint8_t* rec = ((n < 4 || rows) && is_k(y.qkv.t) && d % 256 == 0) ? m.rec : nullptr;
    norm(m.x, y.attn_norm, n, 0, m.h, rec);
    CKL();
    pending_combine = false;
    resid = nullptr;
    if (n >= 4 && ctx->f32_prefill && y.q.t != T_F32) {
      // The reference multiplies q, k and v separately, each on its own
      // 48-row tiles (quant.rs:243): in the exact f32 order the fused
      // matrix would tile rows differently.
      const int64_t width = (int64_t)(m.nh + 2 * m.nkv) * m.hd;
      RC(dense_forward(ctx, y.q, m.h, n, m.qkv, nullptr, width));
      RC(dense_forward(ctx, y.k, m.h, n, m.qkv + y.q.rows, nullptr, width));
      RC(dense_forward(ctx, y.v, m.h, n, m.qkv + y.q.rows + y.k.rows, nullptr, width));
    } else {
      RC(dense_forward(ctx, y.qkv, m.h, n, m.qkv, rec));
    }
    QkPostArgs qa{};
    qa.qkv = m.qkv;
    qa.n = n;
    qa.nh = m.nh;
    qa.nkv = m.nkv;
    qa.hd = m.hd;
    qa.rd = m.rd;
    qa.pos0 = pos0;
    qa.neox = m.arch != KC_ARCH_LLAMA;
    qa.eps = m.eps;
    qa.bq = y.bq;
    qa.bk = y.bk;
    qa.bv = y.bv;
    qa.qn = y.qn;
    qa.kn = y.kn;
    qa.rope = m.rope;
    qa.q_out = m.q;
    const size_t cache_off = (size_t)l * m.n_ctx * m.nkv * m.hd;
    qa.kc = kc0 + cache_off;
    qa.vc = vc0 + cache_off;
    qa.pos_dev = pos_dev;
    qa.row_pos = rows ? m.row_pos : nullptr;
    qa.seq_stride = m.seq_elems();
    launch_qk_post(qa, st);
    CKL();
    launch_attention(m.q, qa.kc, qa.vc, n, m.nh, m.nkv, m.hd, pos0, pos_dev, m.n_ctx, scale, m.att, st, qa.row_pos,
                     qa.seq_stride);
    CKL();
    RC(dense_forward(ctx, y.o, m.att, n, m.tmp));
    resid = m.tmp;
    norm(m.x, y.ffn_norm, n, 0, m.h, nullptr);
    CKL();
    // Router lookahead (transformer.rs:432-436): guess the next streamed
    // layer's experts from this post-attention state and start loading them.
    if (ctx->xs.lookahead && ctx->xs.n_layers > 0 && n <= 4 && l + 1 < m.n_layer) RC(model_lookahead(ctx, m, l, n));
    resid = m.ffn;
    if (!y.gate.w) {  // routed experts (checked in model_finalize)
      const Layer& R = ctx->layers[l];
      const bool defer = ctx->ep.world <= 1 && !R.has_shared;
      bool deferred = false;
      RC(moe_pipeline(ctx, R, R.router, m.h, n, m.ffn, nullptr, nullptr, defer, &deferred));
      if (deferred) {
        pending_combine = true;
        pending_k = R.k;
      }
    } else {
      RC(dense_forward(ctx, y.gate, m.h, n, m.g));
      RC(dense_forward(ctx, y.up, m.h, n, m.u));
      launch_swiglu(m.g, m.u, (int64_t)n * y.gate.rows, st);
      CKL();
      RC(dense_forward(ctx, y.down, m.g, n, m.ffn));
    }
  }
  if (rows) {
    // Every row is its sequence's last token.
    norm(m.x, m.out_norm, n, 0, m.h, nullptr);
    CKL();
    RC(dense_forward(ctx, m.output, m.h, n, m.logits));
    launch_argmax(m.logits, m.n_vocab, m.next, st, n);
    CKL();
    return KC_OK;
  }
  // Final norm of the last row only (transformer.rs:459-466).
  const int64_t last = (int64_t)(n - 1) * d;
  norm(m.x + last, m.out_norm, 1, n - 1, m.h, nullptr);
  CKL();
  RC(dense_forward(ctx, m.output, m.h, 1, m.logits));
  launch_argmax(m.logits, m.n_vocab, m.next, st);
  CKL();
  if (!dev_pos) m.cached += n;
  return KC_OK;
}

int model_forward(kc_ctx* ctx, const uint32_t* tokens, bool tokens_on_dev, int n) {
  Model& m = *ctx->model;
  RC(model_finalize(ctx, m));
  if (n < 1) return fail(ctx, KC_ERR_ARG, "kc_model_forward: forward() needs at least one token");
  if (m.cached + n > m.n_ctx)
    return fail(ctx, KC_ERR_ARG, "kc_model_forward: context full: %d positions needed, n_ctx = %d", m.cached + n,
                m.n_ctx);
  if (!tokens_on_dev)
    for (int i = 0; i < n; ++i)
      if (tokens[i] >= (uint32_t)m.n_vocab)
        return fail(ctx, KC_ERR_ARG, "kc_model_forward: token id %u out of range", tokens[i]);
  for (int c = 0; c < n; c += kModelBatch) {  // n_batch chunks (transformer.rs:293)
    const int nc = std::min(kModelBatch, n - c);
    RC(model_buffers(ctx, m, nc));
    CK(cudaMemcpyAsync(m.tok, tokens + c, (size_t)nc * 4,
                       tokens_on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->stream));
    RC(model_chunk(ctx, m, nc, m.tok, false));
  }
  return KC_OK;
}

// ===========================================================================
extern "C" {

int kc_init(int device, kc_ctx** out) {
  kc_ctx* ctx = nullptr;
  if (!out) return fail(nullptr, KC_ERR_ARG, "kc_init: out is NULL");
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n)
    return fail(nullptr, KC_ERR_CUDA, "kc_init: no CUDA device %d (%d visible)", device, n);
  if (cudaSetDevice(device) != cudaSuccess) return fail(nullptr, KC_ERR_CUDA, "kc_init: cudaSetDevice failed");
  cudaDeviceProp prop;
  cudaGetDeviceProperties(&prop, device);
  if (prop.major < 10) return fail(nullptr, KC_ERR_CUDA, "kc_init: device %d is sm_%d%d, kernels need sm_100a",
                                   device, prop.major, prop.minor);
  ctx = new kc_ctx();
  ctx->device = device;
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->status, sizeof(int)) != cudaSuccess ||
      cudaMemsetAsync(ctx->status, 0, sizeof(int), ctx->stream) != cudaSuccess ||
      cudaHostAlloc(&ctx->status_host, sizeof(int), cudaHostAllocDefault) != cudaSuccess) {
    delete ctx;
    return fail(nullptr, KC_ERR_CUDA, "kc_init: stream/status allocation failed");
  }
  ctx->own_stream = true;
  *out = ctx;
  return KC_OK;
}

void kc_free(kc_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  model_free(ctx);
  ep_free(ctx->ep);
  ep_free_bufs(ctx->epb);
  streams_free(ctx);
  for (auto& [id, L] : ctx->layers) free_layer(L);
  for (auto& [id, D] : ctx->dense) cudaFree(D.w);
  for (auto& r : ctx->prof.recs) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (auto e : ctx->prof.pool) cudaEventDestroy(e);
  cudaFree(ctx->ws.arena);
  cudaFree(ctx->ws_ep.arena);
  cudaFree(ctx->status);
  if (ctx->status_host) cudaFreeHost(ctx->status_host);
  if (ctx->cap) cudaStreamDestroy(ctx->cap);
  if (ctx->aux) {
    cudaStreamSynchronize(ctx->aux);
    cudaStreamDestroy(ctx->aux);
    cudaEventDestroy(ctx->ev_fork);
    cudaEventDestroy(ctx->ev_join);
  }
  if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

const char* kc_last_error(const kc_ctx* ctx) { return ctx ? ctx->err.c_str() : g_init_err.c_str(); }

int kc_set_stream(kc_ctx* ctx, void* s) {
  if (!ctx) return KC_ERR_ARG;
  // NULL is CUDA's legacy default stream, as everywhere in the runtime API.
  if (ctx->own_stream) {
    CK(cudaStreamSynchronize(ctx->stream));
    cudaStreamDestroy(ctx->stream);
    ctx->own_stream = false;
  }
  ctx->stream = static_cast<cudaStream_t>(s);
  ctx->ws.dmeta_n = -1;  // rewritten on the new stream before its next use
  return KC_OK;
}

int kc_reserve(kc_ctx* ctx, int max_tokens) {
  if (!ctx || max_tokens < 0) return KC_ERR_ARG;
  cudaSetDevice(ctx->device);
  int E = 1, K = 1, D = 256, F = 256;
  for (auto& [id, L] : ctx->layers) {
    E = std::max(E, L.n_expert);
    K = std::max(K, L.k);
    D = std::max(D, L.d);
    F = std::max(F, L.ff);
  }
  for (auto& [id, Dn] : ctx->dense) D = std::max<int>(D, (int)Dn.cols);
  return ensure_work(ctx, max_tokens, E, K, D, F);
}

int kc_sync(kc_ctx* ctx) {
  if (!ctx) return KC_ERR_ARG;
  return check_status(ctx);  // synchronises the stream
}

int64_t kc_device_bytes(const kc_ctx* ctx) {
  if (!ctx) return 0;
  const int64_t slots = ctx->xs.arena ? (int64_t)ctx->xs.cache.slots() * ctx->xs.slot_bytes : 0;
  return ctx->weight_bytes + (int64_t)ctx->ws.bytes + (int64_t)ctx->ws_ep.bytes + slots;
}

int kc_upload_experts_range(kc_ctx* ctx, int layer, int n_expert, int first_expert, int n_local, int d, int ff,
                            int t_gate, const void* gate, int t_up, const void* up, int t_down, const void* down,
                            int src_on_device) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!gate || !up || !down || n_expert <= 0 || n_local <= 0 || first_expert < 0 ||
      first_expert + n_local > n_expert || d <= 0 || ff <= 0)
    return fail(ctx, KC_ERR_ARG, "kc_upload_experts: bad arguments");
  if (!type_ok(t_gate) || !type_ok(t_up) || !type_ok(t_down))
    return fail(ctx, KC_ERR_TYPE, "kc_upload_experts: types %d/%d/%d (kernels: Q4_K, Q6_K, Q8_0)", t_gate, t_up,
                t_down);
  if (t_gate != t_up) return fail(ctx, KC_ERR_TYPE, "kc_upload_experts: gate and up types differ");
  if (d % block_elems(t_gate) || ff % block_elems(t_down))
    return fail(ctx, KC_ERR_SHAPE, "kc_upload_experts: d=%d / ff=%d not a block multiple", d, ff);
  if (d % 256 || ff % 32) return fail(ctx, KC_ERR_SHAPE, "kc_upload_experts: d must be a multiple of 256");
  cudaSetDevice(ctx->device);
  RC(wait_device_source(ctx, src_on_device != 0));
  Layer& L = ctx->layers[layer];
  RC(drop_streamed(ctx, L));
  cudaFree(L.gate);
  cudaFree(L.up);
  cudaFree(L.down);
  L.gate = L.up = L.down = nullptr;
  L.has_experts = false;
  L.id = layer;
  if (L.has_router && L.n_expert != n_expert)
    return fail(ctx, KC_ERR_SHAPE, "kc_upload_experts: %d experts but the router has %d", n_expert, L.n_expert);
  L.n_expert = n_expert;
  L.first_expert = first_expert;
  L.n_local = n_local;
  L.d = d;
  L.ff = ff;
  L.t_gate = t_gate;
  L.t_up = t_up;
  L.t_down = t_down;
  L.mb_gate = dev_matrix_bytes(t_gate, ff, d);
  L.mb_down = dev_matrix_bytes(t_down, d, ff);
  const int64_t gbytes = (int64_t)n_local * L.mb_gate, dbytes = (int64_t)n_local * L.mb_down;
  CK(cudaMalloc(&L.gate, gbytes));
  CK(cudaMalloc(&L.up, gbytes));
  CK(cudaMalloc(&L.down, dbytes));
  ctx->weight_bytes += 2 * gbytes + dbytes;
  RC(upload_matrix(ctx, t_gate, gate, n_local, ff, d, L.gate, src_on_device != 0));
  RC(upload_matrix(ctx, t_up, up, n_local, ff, d, L.up, src_on_device != 0));
  RC(upload_matrix(ctx, t_down, down, n_local, d, ff, L.down, src_on_device != 0));
  CK(cudaStreamSynchronize(ctx->stream));
  L.has_experts = true;
  return KC_OK;
}

int kc_upload_experts(kc_ctx* ctx, int layer, int n_expert, int d, int ff, int t_gate, const void* gate, int t_up,
                      const void* up, int t_down, const void* down, int src_on_device) {
  return kc_upload_experts_range(ctx, layer, n_expert, 0, n_expert, d, ff, t_gate, gate, t_up, up, t_down, down,
                                 src_on_device);
}

int kc_upload_experts_streamed(kc_ctx* ctx, int layer, int n_expert, int d, int ff, int t_gate, const void* gate,
                               int t_up, const void* up, int t_down, const void* down, int src_on_device) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!gate || !up || !down || n_expert <= 0 || d <= 0 || ff <= 0)
    return fail(ctx, KC_ERR_ARG, "kc_upload_experts_streamed: bad arguments");
  if (!type_ok(t_gate) || !type_ok(t_up) || !type_ok(t_down))
    return fail(ctx, KC_ERR_TYPE, "kc_upload_experts_streamed: types %d/%d/%d (kernels: Q4_K, Q6_K, Q8_0)",
                t_gate, t_up, t_down);
  if (t_gate != t_up) return fail(ctx, KC_ERR_TYPE, "kc_upload_experts_streamed: gate and up types differ");
  if (d % block_elems(t_gate) || ff % block_elems(t_down) || d % 256 || ff % 32)
    return fail(ctx, KC_ERR_SHAPE, "kc_upload_experts_streamed: d=%d / ff=%d (d %% 256 == 0, ff %% 32 == 0)", d,
                ff);
  if (ctx->ep.world > 1)
    return fail(ctx, KC_ERR_STATE, "kc_upload_experts_streamed: not served by expert parallelism");
  cudaSetDevice(ctx->device);
  RC(wait_device_source(ctx, src_on_device != 0));
  ExpertStreams& S = ctx->xs;
  Layer& L = ctx->layers[layer];
  if (L.has_router && L.n_expert != n_expert)
    return fail(ctx, KC_ERR_SHAPE, "kc_upload_experts_streamed: %d experts but the router has %d", n_expert,
                L.n_expert);
  // One expert's gate, up and down side by side, each 256-byte aligned: one
  // copy per expert, and the kernels' bulk copies stay 16-byte aligned.
  const int64_t mb_gate = dev_matrix_bytes(t_gate, ff, d), mb_down = dev_matrix_bytes(t_down, d, ff);
  auto al256 = [](int64_t v) { return (v + 255) / 256 * 256; };
  const int64_t up_off = al256(mb_gate), down_off = up_off + al256(mb_gate), slot_bytes = down_off + al256(mb_down);
  const int others = S.n_layers - (L.streamed ? 1 : 0);
  if (others > 0 && S.slot_bytes != slot_bytes)
    return fail(ctx, KC_ERR_SHAPE,
                "kc_upload_experts_streamed: every host-streamed layer shares the slots' shape (%lld bytes per "
                "expert), layer %d needs %lld",
                (long long)S.slot_bytes, layer, (long long)slot_bytes);
  RC(drop_streamed(ctx, L));
  cudaFree(L.gate);
  cudaFree(L.up);
  cudaFree(L.down);
  L.gate = L.up = L.down = nullptr;
  L.has_experts = false;
  if (S.slot_bytes != slot_bytes) {  // new slot shape: the arena is made again at first use
    RC(streams_invalidate(ctx));
    cudaFree(S.arena);
    S.arena = nullptr;
    S.slot_bytes = slot_bytes;
  }
  L.id = layer;
  L.n_expert = n_expert;
  L.first_expert = 0;
  L.n_local = n_expert;
  L.d = d;
  L.ff = ff;
  L.t_gate = t_gate;
  L.t_up = t_up;
  L.t_down = t_down;
  L.mb_gate = mb_gate;
  L.mb_down = mb_down;
  L.up_off = up_off;
  L.down_off = down_off;
  L.slot_bytes = slot_bytes;
  if (cudaHostAlloc(&L.host, (size_t)n_expert * slot_bytes, cudaHostAllocDefault) != cudaSuccess) {
    cudaGetLastError();
    L.host = nullptr;
    return fail(ctx, KC_ERR_OOM, "kc_upload_experts_streamed: %lld bytes of pinned host memory",
                (long long)n_expert * slot_bytes);
  }
  // Convert a chunk of experts at a time into the device layout on the GPU,
  // then read it back beside the other matrices of each expert.
  const int64_t chunk = std::max<int64_t>(1, std::min<int64_t>(n_expert, (256ll << 20) / slot_bytes));
  uint8_t* tmp = nullptr;
  CK(cudaMalloc(&tmp, (size_t)chunk * std::max(mb_gate, mb_down)));
  int rc = KC_OK;
  struct Part {
    int t;
    const void* src;
    int64_t rows, cols, mb, off;
  } parts[3] = {{t_gate, gate, ff, d, mb_gate, 0}, {t_up, up, ff, d, mb_gate, up_off},
                {t_down, down, d, ff, mb_down, down_off}};
  for (int64_t e0 = 0; e0 < n_expert && rc == KC_OK; e0 += chunk) {
    const int64_t ne = std::min<int64_t>(chunk, n_expert - e0);
    for (const Part& p : parts) {
      const int64_t mat_src = p.rows * gguf_row_bytes(p.t, p.cols);
      rc = upload_matrix(ctx, p.t, static_cast<const uint8_t*>(p.src) + e0 * mat_src, ne, p.rows, p.cols, tmp,
                         src_on_device != 0);
      if (rc != KC_OK) break;
      cudaError_t e = cudaMemcpy2DAsync(L.host + e0 * slot_bytes + p.off, (size_t)slot_bytes, tmp, (size_t)p.mb,
                                        (size_t)p.mb, (size_t)ne, cudaMemcpyDeviceToHost, ctx->stream);
      if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
      if (e != cudaSuccess) {
        rc = fail(ctx, KC_ERR_CUDA, "kc_upload_experts_streamed: %s", cudaGetErrorString(e));
        break;
      }
    }
  }
  cudaFree(tmp);
  if (rc != KC_OK) {
    cudaFreeHost(L.host);
    L.host = nullptr;
    return rc;
  }
  L.streamed = true;
  L.has_experts = true;
  ++S.n_layers;
  return KC_OK;
}

int kc_expert_cache_reserve(kc_ctx* ctx, int capacity, int scratch, int spec, int policy) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (capacity < 0 || scratch < 0 || spec < 0 || capacity + scratch < 1 ||
      (policy != KC_EXPERT_POLICY_LFRU && policy != KC_EXPERT_POLICY_LRU))
    return fail(ctx, KC_ERR_ARG, "kc_expert_cache_reserve: capacity %d, scratch %d, spec %d, policy %d", capacity,
                scratch, spec, policy);
  cudaSetDevice(ctx->device);
  ExpertStreams& S = ctx->xs;
  RC(streams_invalidate(ctx));
  cudaFree(S.arena);
  S.arena = nullptr;
  while ((int)S.ready.size() > capacity + scratch + spec) {
    cudaEventDestroy(S.ready.back());
    S.ready.pop_back();
  }
  S.capacity = capacity;
  S.scratch = scratch;
  S.spec = spec;
  S.policy = policy == KC_EXPERT_POLICY_LRU ? ExpertPolicy::Lru : ExpertPolicy::Lfru;
  S.cache.configure(capacity, scratch, spec, S.policy);
  // With a streamed layer already uploaded the slots are made now, so that a
  // reservation HBM cannot hold fails here rather than in a later call.
  if (S.slot_bytes) RC(streams_alloc(ctx, capacity));
  return KC_OK;
}

int kc_expert_prefetch(kc_ctx* ctx, int layer, const int32_t* experts, int n) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  auto it = ctx->layers.find(layer);
  if (it == ctx->layers.end() || !it->second.streamed)
    return fail(ctx, KC_ERR_STATE, "kc_expert_prefetch: layer %d has no host-streamed experts", layer);
  const Layer& L = it->second;
  if (n < 0 || (n > 0 && !experts)) return fail(ctx, KC_ERR_ARG, "kc_expert_prefetch: bad arguments");
  std::vector<char> seen(L.n_expert, 0);
  for (int i = 0; i < n; ++i) {
    if (experts[i] < 0 || experts[i] >= L.n_expert)
      return fail(ctx, KC_ERR_ARG, "kc_expert_prefetch: expert %d of %d", experts[i], L.n_expert);
    seen[experts[i]] = 1;
  }
  std::vector<int> list;
  for (int e = 0; e < L.n_expert; ++e)
    if (seen[e]) list.push_back(e);
  cudaSetDevice(ctx->device);
  return streams_prefetch(ctx, L, list);
}

int kc_expert_cache_stats(const kc_ctx* ctx, uint64_t* out, int n) {
  if (!ctx || n < 0 || (n > 0 && !out)) return KC_ERR_ARG;
  const ExpertStreams& S = ctx->xs;
  const ExpertCacheStats& c = S.cache.stats();
  const uint64_t v[KC_XS_N] = {(uint64_t)std::max(0, S.capacity), (uint64_t)S.cache.cached(), c.requests, c.hits,
                               c.late, c.misses, c.scratch_loads, c.bytes_read, c.prefetch_issued, c.prefetch_used,
                               c.prefetch_wasted, c.evictions, c.lookahead_predicted, c.lookahead_correct, c.reads,
                               c.forced, (uint64_t)std::max(0, S.scratch), (uint64_t)std::max(0, S.spec),
                               c.spec_pauses};
  for (int i = 0; i < n; ++i) out[i] = i < KC_XS_N ? v[i] : 0;
  return KC_OK;
}

int kc_expert_cache_decay(kc_ctx* ctx) {
  if (!ctx) return KC_ERR_ARG;
  ctx->xs.cache.decay();
  return KC_OK;
}

int kc_upload_router(kc_ctx* ctx, int layer, const float* router_w, int n_expert, int d, int k, int norm_topk,
                     float weights_scale, int src_on_device) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!router_w || n_expert <= 0 || d <= 0 || k < 1 || k > 64 || k > n_expert || n_expert > 1024)
    return fail(ctx, KC_ERR_ARG, "kc_upload_router: bad arguments (E=%d d=%d k=%d; k <= 64, E <= 1024)",
                n_expert, d, k);
  cudaSetDevice(ctx->device);
  RC(wait_device_source(ctx, src_on_device != 0));
  Layer& L = ctx->layers[layer];
  if (L.has_experts && (L.n_expert != n_expert || L.d != d))
    return fail(ctx, KC_ERR_SHAPE, "kc_upload_router: shape [%d, %d] does not match the experts [%d, %d]",
                n_expert, d, L.n_expert, L.d);
  cudaFree(L.router);
  L.router = nullptr;
  CK(cudaMalloc(&L.router, (size_t)n_expert * d * 4));
  CK(cudaMemcpyAsync(L.router, router_w, (size_t)n_expert * d * 4,
                     src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));
  ctx->weight_bytes += (int64_t)n_expert * d * 4;
  L.has_router = true;
  L.n_expert = n_expert;
  L.d = d;
  L.k = k;
  L.norm_topk = norm_topk ? 1 : 0;
  L.weights_scale = weights_scale;
  return KC_OK;
}

int kc_upload_dense(kc_ctx* ctx, int tensor_id, int t, const void* w, int64_t rows, int64_t cols,
                    int src_on_device) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!w || rows <= 0 || cols <= 0) return fail(ctx, KC_ERR_ARG, "kc_upload_dense: bad arguments");
  if (!type_ok(t) && t != T_F32) return fail(ctx, KC_ERR_TYPE, "kc_upload_dense: type %d has no kernel", t);
  if (cols % block_elems(t)) return fail(ctx, KC_ERR_SHAPE, "kc_upload_dense: cols %lld", (long long)cols);
  cudaSetDevice(ctx->device);
  RC(wait_device_source(ctx, src_on_device != 0));
  Dense& D = ctx->dense[tensor_id];
  cudaFree(D.w);
  D.t = t;
  D.rows = rows;
  D.cols = cols;
  D.rs = round16(cols * 4);
  const int64_t bytes = dev_matrix_bytes(t, rows, cols);
  CK(cudaMalloc(&D.w, bytes));
  ctx->weight_bytes += bytes;
  RC(upload_matrix(ctx, t, w, 1, rows, cols, D.w, src_on_device != 0));
  CK(cudaStreamSynchronize(ctx->stream));
  return KC_OK;
}

int kc_upload_shared_expert(kc_ctx* ctx, int layer, int ff_shared, int d, int t_gate, const void* gate, int t_up,
                            const void* up, int t_down, const void* down, const float* gate_inp,
                            int src_on_device) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!gate || !up || !down || ff_shared <= 0 || d <= 0)
    return fail(ctx, KC_ERR_ARG, "kc_upload_shared_expert: bad arguments");
  for (int t : {t_gate, t_up, t_down})
    if (!type_ok(t)) return fail(ctx, KC_ERR_TYPE, "kc_upload_shared_expert: type %d has no kernel", t);
  if (d % block_elems(t_gate) || d % block_elems(t_up) || ff_shared % block_elems(t_down) || d % 256 ||
      ff_shared % 32)
    return fail(ctx, KC_ERR_SHAPE, "kc_upload_shared_expert: d=%d / ff=%d do not fit the block sizes", d,
                ff_shared);
  cudaSetDevice(ctx->device);
  RC(wait_device_source(ctx, src_on_device != 0));
  Layer& L = ctx->layers[layer];
  if (L.has_experts && L.d != d) return fail(ctx, KC_ERR_SHAPE, "kc_upload_shared_expert: d differs from the layer's");
  const struct {
    Layer::Mat* m;
    int t;
    const void* src;
    int64_t rows, cols;
  } mats[3] = {{&L.sh_gate, t_gate, gate, ff_shared, d}, {&L.sh_up, t_up, up, ff_shared, d},
               {&L.sh_down, t_down, down, d, ff_shared}};
  for (const auto& x : mats) {
    cudaFree(x.m->w);
    x.m->w = nullptr;
    x.m->t = x.t;
    x.m->rows = x.rows;
    x.m->cols = x.cols;
    const int64_t bytes = dev_matrix_bytes(x.t, x.rows, x.cols);
    CK(cudaMalloc(&x.m->w, bytes));
    ctx->weight_bytes += bytes;
    RC(upload_matrix(ctx, x.t, x.src, 1, x.rows, x.cols, x.m->w, src_on_device != 0));
  }
  cudaFree(L.sh_inp);
  L.sh_inp = nullptr;
  if (gate_inp) {
    CK(cudaMalloc(&L.sh_inp, (size_t)d * 4));
    CK(cudaMemcpyAsync(L.sh_inp, gate_inp, (size_t)d * 4, src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                       ctx->stream));
  }
  L.sh_ff = ff_shared;
  L.d = d;
  L.has_shared = true;
  CK(cudaStreamSynchronize(ctx->stream));
  return KC_OK;
}

int kc_moe_ffn_dev(kc_ctx* ctx, int layer, const float* h, int n_tok, float* out, int32_t* topk_ids,
                   float* topk_w) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  auto it = ctx->layers.find(layer);
  if (it == ctx->layers.end() || !it->second.has_experts || !it->second.has_router)
    return fail(ctx, KC_ERR_STATE, "kc_moe_ffn: layer %d has no uploaded experts and router", layer);
  if (n_tok < 0 || (n_tok > 0 && (!h || !out))) return fail(ctx, KC_ERR_ARG, "kc_moe_ffn: bad buffers");
  const Layer& L = it->second;
  if (ctx->ep.world <= 1 && L.n_local != L.n_expert)
    return fail(ctx, KC_ERR_STATE, "kc_moe_ffn: layer %d holds a shard of the experts but no expert-parallel "
                                   "group was joined (kc_ep_init)", layer);
  cudaSetDevice(ctx->device);
  return moe_pipeline(ctx, L, L.router, h, n_tok, out, topk_ids, topk_w);
}

int kc_moe_ffn(kc_ctx* ctx, int layer, const float* h, int n_tok, const float* router_w, int n_expert, int k,
               int norm_topk, float weights_scale, float* out, int32_t* topk_ids, float* topk_w) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  auto it = ctx->layers.find(layer);
  if (it == ctx->layers.end() || !it->second.has_experts)
    return fail(ctx, KC_ERR_STATE, "kc_moe_ffn: layer %d has no uploaded experts", layer);
  if (n_tok < 0 || (n_tok > 0 && (!h || !out))) return fail(ctx, KC_ERR_ARG, "kc_moe_ffn: bad buffers");
  cudaSetDevice(ctx->device);
  Layer L = it->second;
  if (router_w) {
    if (n_expert != L.n_expert || k < 1 || k > 64 || k > n_expert)
      return fail(ctx, KC_ERR_ARG, "kc_moe_ffn: router [%d] / k=%d do not fit the layer's %d experts", n_expert,
                  k, L.n_expert);
    L.k = k;
    L.norm_topk = norm_topk ? 1 : 0;
    L.weights_scale = weights_scale;
  } else if (!L.has_router) {
    return fail(ctx, KC_ERR_STATE, "kc_moe_ffn: no router uploaded for layer %d and none given", layer);
  }
  if (ctx->ep.world <= 1 && L.n_local != L.n_expert)
    return fail(ctx, KC_ERR_STATE, "kc_moe_ffn: layer %d holds a shard of the experts", layer);
  RC(ensure_work(ctx, n_tok, L.n_expert, L.k, layer_work_d(L), layer_work_f(L)));
  Work& W = ctx->ws;
  const float* router = L.router;
  if (router_w) {
    CK(cudaMemcpyAsync(W.router_tmp, router_w, (size_t)L.n_expert * L.d * 4, cudaMemcpyHostToDevice,
                       ctx->stream));
    router = W.router_tmp;
  }
  if (n_tok > 0) CK(cudaMemcpyAsync(W.h_in, h, (size_t)n_tok * L.d * 4, cudaMemcpyHostToDevice, ctx->stream));
  // ids / w land in the workspace; copied out below.
  RC(moe_pipeline(ctx, L, router, W.h_in, n_tok, W.out, nullptr, nullptr));
  if (n_tok > 0) CK(cudaMemcpyAsync(out, W.out, (size_t)n_tok * L.d * 4, cudaMemcpyDeviceToHost, ctx->stream));
  const bool ep = ctx->ep.world > 1;
  if (topk_ids && n_tok > 0)
    CK(cudaMemcpyAsync(topk_ids, ep ? ctx->epb.ids_home : W.ids, (size_t)n_tok * L.k * 4, cudaMemcpyDeviceToHost,
                       ctx->stream));
  if (topk_w && n_tok > 0)
    CK(cudaMemcpyAsync(topk_w, ep ? ctx->epb.w_home : W.w, (size_t)n_tok * L.k * 4, cudaMemcpyDeviceToHost,
                       ctx->stream));
  return check_status(ctx);  // synchronises the stream
}

int kc_matmul_dev(kc_ctx* ctx, int tensor_id, const float* x, int n, float* out) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  auto it = ctx->dense.find(tensor_id);
  if (it == ctx->dense.end()) return fail(ctx, KC_ERR_STATE, "kc_matmul: tensor %d not uploaded", tensor_id);
  if (n < 0 || (n > 0 && (!x || !out))) return fail(ctx, KC_ERR_ARG, "kc_matmul: bad buffers");
  const Dense& D = it->second;
  cudaSetDevice(ctx->device);
  if (n == 0) return KC_OK;
  return dense_forward(ctx, D, x, n, out);
}

int kc_matmul(kc_ctx* ctx, int tensor_id, const float* x, int n, float* out) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  auto it = ctx->dense.find(tensor_id);
  if (it == ctx->dense.end()) return fail(ctx, KC_ERR_STATE, "kc_matmul: tensor %d not uploaded", tensor_id);
  if (n <= 0) return n == 0 ? KC_OK : fail(ctx, KC_ERR_ARG, "kc_matmul: n < 0");
  const Dense D = it->second;
  cudaSetDevice(ctx->device);
  // Stage x and out in the workspace's h_in/out buffers.
  RC(ensure_work(ctx, n, 1, 1, (int)std::max(D.cols, D.rows), 256));
  Work& W = ctx->ws;
  CK(cudaMemcpyAsync(W.h_in, x, (size_t)n * D.cols * 4, cudaMemcpyHostToDevice, ctx->stream));
  RC(kc_matmul_dev(ctx, tensor_id, W.h_in, n, W.out));
  CK(cudaMemcpyAsync(out, W.out, (size_t)n * D.rows * 4, cudaMemcpyDeviceToHost, ctx->stream));
  return check_status(ctx);  // synchronises the stream
}

int kc_q8k_quantize_dev(kc_ctx* ctx, const float* x, int64_t n_rows, int64_t cols, int8_t* q, float* d,
                        int32_t* bsums) {
  if (!ctx) return KC_ERR_ARG;
  if (cols % 256) return fail(ctx, KC_ERR_SHAPE, "kc_q8k_quantize: cols %% 256 != 0");
  cudaSetDevice(ctx->device);
  launch_q8k_quantize(x, nullptr, n_rows, cols, q, d, bsums, ctx->stream);
  CKL();
  return KC_OK;
}

int kc_q8_quantize_dev(kc_ctx* ctx, const float* x, int64_t n_rows, int64_t cols, int8_t* q, float* d,
                       int32_t* s16) {
  if (!ctx) return KC_ERR_ARG;
  if (cols % 32) return fail(ctx, KC_ERR_SHAPE, "kc_q8_quantize: cols %% 32 != 0");
  cudaSetDevice(ctx->device);
  launch_q8_quantize(x, nullptr, n_rows, cols, q, d, s16, ctx->stream);
  CKL();
  return KC_OK;
}

int kc_route_dev(kc_ctx* ctx, const float* logits, int n_tok, int n_expert, int k, int norm_topk,
                 float weights_scale, int32_t* ids, float* w) {
  if (!ctx) return KC_ERR_ARG;
  if (k < 1 || k > 64 || k > n_expert || n_expert > 1024) return fail(ctx, KC_ERR_ARG, "kc_route: bad k/E");
  cudaSetDevice(ctx->device);
  launch_route(logits, n_tok, n_expert, k, norm_topk, weights_scale, ids, w, ctx->stream);
  CKL();
  return KC_OK;
}

int kc_router_logits_dev(kc_ctx* ctx, const float* router_w, int n_expert, int d, const float* h, int n_tok,
                         float* logits) {
  if (!ctx) return KC_ERR_ARG;
  cudaSetDevice(ctx->device);
  launch_router_logits(router_w, d, n_expert, d, h, n_tok, logits, ctx->status, ctx->stream);
  CKL();
  return KC_OK;
}

int kc_block_sums_dev(kc_ctx* ctx, int t, const void* w, int64_t rows, int64_t cols, const int8_t* q,
                      const int32_t* bsums, int n_act, int32_t* out) {
  if (!ctx) return KC_ERR_ARG;
  if (!is_k(t)) return fail(ctx, KC_ERR_TYPE, "kc_block_sums: K-quant types only");
  if (cols % 256) return fail(ctx, KC_ERR_SHAPE, "kc_block_sums: cols %% 256 != 0");
  cudaSetDevice(ctx->device);
  launch_block_sums(t, w, rows, cols, q, bsums, n_act, out, ctx->stream);
  CKL();
  return KC_OK;
}

int kc_quantize_dev(kc_ctx* ctx, int t, const float* x, int64_t rows, int64_t cols, void* out) {
  if (!ctx) return KC_ERR_ARG;
  cudaSetDevice(ctx->device);
  int rc = launch_quantize(t, x, rows, cols, out, ctx->stream);
  if (rc != KC_OK) return fail(ctx, rc, "kc_quantize: type %d cols %lld", t, (long long)cols);
  CKL();
  return KC_OK;
}

int kc_profile_enable(kc_ctx* ctx, int on) {
  if (!ctx) return KC_ERR_ARG;
  ctx->prof.on = on != 0;
  return KC_OK;
}

int64_t kc_kernel_launches(void) { return kc::g_kernel_launches.load(std::memory_order_relaxed); }

int kc_profile_read(kc_ctx* ctx, double* stage_ms, int64_t* stage_calls, int n_stages) {
  if (!ctx || n_stages < 0) return KC_ERR_ARG;
  cudaSetDevice(ctx->device);
  CK(cudaStreamSynchronize(ctx->stream));
  for (int i = 0; i < n_stages; ++i) {
    if (stage_ms) stage_ms[i] = 0;
    if (stage_calls) stage_calls[i] = 0;
  }
  for (auto& r : ctx->prof.recs) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.a, r.b);
    if (r.stage < n_stages) {
      if (stage_ms) stage_ms[r.stage] += ms;
      if (stage_calls) stage_calls[r.stage] += 1;
    }
    ctx->prof.pool.push_back(r.a);
    ctx->prof.pool.push_back(r.b);
  }
  ctx->prof.recs.clear();
  return KC_OK;
}

int kc_ep_unique_id(char out[128]) { return ep_unique_id(out); }

int kc_ep_init(kc_ctx* ctx, int rank, int world, const char uid[128]) {
  if (!ctx) return KC_ERR_ARG;
  cudaSetDevice(ctx->device);
  int rc = ep_init(ctx->ep, rank, world, uid);
  if (rc != KC_OK) return fail(ctx, rc, "kc_ep_init: %s", ep_last_error(ctx->ep));
  return KC_OK;
}

int kc_ep_reserve(kc_ctx* ctx, int max_tokens) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (ctx->ep.world < 2) return fail(ctx, KC_ERR_STATE, "kc_ep_reserve: join an expert-parallel group first");
  int d = 0, k = 0;
  for (const auto& [id, L] : ctx->layers)
    if (L.has_experts) {
      d = std::max(d, L.d);
      k = std::max(k, L.k);
    }
  if (d == 0 || k == 0) return fail(ctx, KC_ERR_STATE, "kc_ep_reserve: upload the layers and routers first");
  cudaSetDevice(ctx->device);
  CK(cudaStreamSynchronize(ctx->stream));
  const int rc = ep_p2p_setup(ctx->ep, max_tokens, d, k, ctx->stream);
  if (rc != KC_OK) return fail(ctx, rc, "kc_ep_reserve: %s", ep_last_error(ctx->ep));
  return KC_OK;
}

// ---- whole model (dense decode path) ---------------------------------------
int kc_set_option(kc_ctx* ctx, int option, int value) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (option == KC_OPT_F32_PREFILL) {
    ctx->f32_prefill = value != 0;
    return KC_OK;
  }
  if (option == KC_OPT_LOOKAHEAD) {
    ctx->xs.lookahead = value != 0;
    return KC_OK;
  }

  return fail(ctx, KC_ERR_ARG, "kc_set_option: unknown option %d", option);
}

int kc_model_init(kc_ctx* ctx, int n_layer, int d, int n_head, int n_head_kv, int head_dim, int n_vocab, int n_ctx,
                  int rope_dim, float rope_base, float rms_eps, int arch) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (n_layer < 1 || d < 1 || d % 4 || n_head < 1 || n_head_kv < 1 || n_head % n_head_kv || head_dim < 1 ||
      head_dim > 256 || head_dim % 8 || n_vocab < 1 || n_ctx < 1 || n_ctx > attention_max_positions(head_dim) ||
      rope_dim < 0 || rope_dim > head_dim || rope_dim % 2 ||
      arch < KC_ARCH_LLAMA || arch > KC_ARCH_QWEN3)
    return fail(ctx, KC_ERR_ARG, "kc_model_init: bad hyper-parameters");
  cudaSetDevice(ctx->device);
  CK(cudaStreamSynchronize(ctx->stream));
  model_free(ctx);
  // The new model's routed layers are uploaded after this call under indices
  // 0 .. n_layer-1: drop what an earlier model left there.
  for (auto it = ctx->layers.begin(); it != ctx->layers.end();) {
    if (it->first >= 0 && it->first < n_layer) {
      if (it->second.streamed) {
        streams_invalidate(ctx);
        --ctx->xs.n_layers;
      }
      free_layer(it->second);
      it = ctx->layers.erase(it);
    } else {
      ++it;
    }
  }
  Model* m = new Model();
  ctx->model = m;
  m->n_layer = n_layer; m->d = d; m->nh = n_head; m->nkv = n_head_kv; m->hd = head_dim; m->n_vocab = n_vocab;
  m->n_ctx = n_ctx; m->rd = rope_dim; m->rope_base = rope_base; m->eps = rms_eps; m->arch = arch;
  m->L.resize(n_layer);
  const size_t cache = (size_t)n_layer * n_ctx * n_head_kv * head_dim;
  CK(cudaMalloc(&m->kc, cache * 2));
  CK(cudaMalloc(&m->vc, cache * 2));
  CK(cudaMemsetAsync(m->kc, 0, cache * 2, ctx->stream));
  CK(cudaMemsetAsync(m->vc, 0, cache * 2, ctx->stream));
  // RoPE angles on the host with the C library's powf / sinf / cosf, as Rust's
  // f32::powf / sin_cos call them (transformer.rs:248, 350).
  const int half = std::max(1, rope_dim / 2);
  std::vector<float> inv(half);
  for (int i = 0; i < rope_dim / 2; ++i) inv[i] = std::pow(rope_base, -(2.0f * (float)i) / (float)rope_dim);
  std::vector<float2> tab((size_t)n_ctx * half);
  for (int p = 0; p < n_ctx; ++p)
    for (int i = 0; i < rope_dim / 2; ++i) {
      const float a = (float)p * inv[i];
      tab[(size_t)p * half + i] = make_float2(std::sin(a), std::cos(a));
    }
  CK(cudaMalloc(&m->rope, tab.size() * sizeof(float2)));
  // On the context's stream, waited for here: tab is a host temporary.
  CK(cudaMemcpyAsync(m->rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice, ctx->stream));
  CK(cudaStreamSynchronize(ctx->stream));
  CK(cudaMalloc(&m->logits, (size_t)n_vocab * 4));
  CK(cudaMalloc(&m->next, 4));
  CK(cudaMalloc(&m->counters, 2 * sizeof(int)));
  m->bytes = (int64_t)cache * 4 + (int64_t)tab.size() * 8;
  return KC_OK;
}

int kc_model_tensor(kc_ctx* ctx, int layer, int kind, int t, const void* w, int64_t rows, int64_t cols,
                    int src_on_device) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  Model* m = ctx->model;
  if (!m) return fail(ctx, KC_ERR_STATE, "kc_model_tensor: call kc_model_init first");
  if (!w || rows < 1 || cols < 1) return fail(ctx, KC_ERR_ARG, "kc_model_tensor: bad arguments");
  if (!type_ok(t) && t != T_F32) return fail(ctx, KC_ERR_TYPE, "kc_model_tensor: type %d has no kernel", t);
  if (cols % block_elems(t)) return fail(ctx, KC_ERR_SHAPE, "kc_model_tensor: cols %lld", (long long)cols);
  cudaSetDevice(ctx->device);
  RC(wait_device_source(ctx, src_on_device != 0));
  const bool on_dev = src_on_device != 0;
  m->ready = false;
  if (layer < 0) {
    switch (kind) {
      case KC_T_TOKEN_EMBD:
        if (cols != m->d || rows != m->n_vocab) return fail(ctx, KC_ERR_SHAPE, "kc_model_tensor: embedding shape");
        cudaFree(m->embd);
        m->embd_t = t;
        m->embd_rb = gguf_row_bytes(t, cols);
        CK(cudaMalloc(&m->embd, rows * m->embd_rb));
        CK(cudaMemcpyAsync(m->embd, w, rows * m->embd_rb, on_dev ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                           ctx->stream));
        CK(cudaStreamSynchronize(ctx->stream));
        return KC_OK;
      case KC_T_OUTPUT_NORM:
        if (t != T_F32 || rows * cols != m->d) return fail(ctx, KC_ERR_SHAPE, "kc_model_tensor: output norm");
        RC(model_vec(ctx, m->out_norm, w, m->d, on_dev));
        break;
      case KC_T_OUTPUT:
        if (cols != m->d || rows != m->n_vocab) return fail(ctx, KC_ERR_SHAPE, "kc_model_tensor: output shape");
        RC(model_dense(ctx, m->output, t, w, rows, cols, on_dev));
        break;
      default:
        return fail(ctx, KC_ERR_ARG, "kc_model_tensor: unknown model tensor kind %d", kind);
    }
    CK(cudaStreamSynchronize(ctx->stream));
    return KC_OK;
  }
  if (layer >= m->n_layer) return fail(ctx, KC_ERR_ARG, "kc_model_tensor: layer %d of %d", layer, m->n_layer);
  Model::Lay& y = m->L[layer];
  const int64_t n = rows * cols;
  auto vec = [&](float*& dst, int64_t expect) -> int {
    if (t != T_F32 || n != expect) return fail(ctx, KC_ERR_SHAPE, "kc_model_tensor: vector kind %d", kind);
    return model_vec(ctx, dst, w, n, on_dev);
  };
  switch (kind) {
    case KC_T_ATTN_NORM: RC(vec(y.attn_norm, m->d)); break;
    case KC_T_FFN_NORM: RC(vec(y.ffn_norm, m->d)); break;
    case KC_T_ATTN_Q_NORM: RC(vec(y.qn, m->hd)); break;
    case KC_T_ATTN_K_NORM: RC(vec(y.kn, m->hd)); break;
    case KC_T_ATTN_Q_BIAS: RC(vec(y.bq, (int64_t)m->nh * m->hd)); break;
    case KC_T_ATTN_K_BIAS: RC(vec(y.bk, (int64_t)m->nkv * m->hd)); break;
    case KC_T_ATTN_V_BIAS: RC(vec(y.bv, (int64_t)m->nkv * m->hd)); break;
    case KC_T_ATTN_Q: RC(model_dense(ctx, y.q, t, w, rows, cols, on_dev)); break;
    case KC_T_ATTN_K: RC(model_dense(ctx, y.k, t, w, rows, cols, on_dev)); break;
    case KC_T_ATTN_V: RC(model_dense(ctx, y.v, t, w, rows, cols, on_dev)); break;
    case KC_T_ATTN_OUT: RC(model_dense(ctx, y.o, t, w, rows, cols, on_dev)); break;
    case KC_T_FFN_GATE: RC(model_dense(ctx, y.gate, t, w, rows, cols, on_dev)); break;
    case KC_T_FFN_UP: RC(model_dense(ctx, y.up, t, w, rows, cols, on_dev)); break;
    case KC_T_FFN_DOWN: RC(model_dense(ctx, y.down, t, w, rows, cols, on_dev)); break;
    default: return fail(ctx, KC_ERR_ARG, "kc_model_tensor: unknown layer tensor kind %d", kind);
  }
  CK(cudaStreamSynchronize(ctx->stream));
  return KC_OK;
}

int kc_model_forward(kc_ctx* ctx, const uint32_t* tokens, int n, float* logits, uint32_t* next_token) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!ctx->model) return fail(ctx, KC_ERR_STATE, "kc_model_forward: call kc_model_init first");
  if (!tokens) return fail(ctx, KC_ERR_ARG, "kc_model_forward: tokens is NULL");
  cudaSetDevice(ctx->device);
  Model& m = *ctx->model;
  if (!m.seq_pos.empty()) m.seq_pos[0] = -1;  // sequence 0 loses its pending token
  RC(model_forward(ctx, tokens, false, n));
  if (logits) CK(cudaMemcpyAsync(logits, m.logits, (size_t)m.n_vocab * 4, cudaMemcpyDeviceToHost, ctx->stream));
  if (next_token) CK(cudaMemcpyAsync(next_token, m.next, 4, cudaMemcpyDeviceToHost, ctx->stream));
  return check_status(ctx);  // synchronises the stream
}

int kc_model_generate(kc_ctx* ctx, const uint32_t* prompt, int n_prompt, int n_gen, uint32_t* out_tokens) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!ctx->model) return fail(ctx, KC_ERR_STATE, "kc_model_generate: call kc_model_init first");
  if (!prompt || n_prompt < 1 || n_gen < 0 || (n_gen > 0 && !out_tokens))
    return fail(ctx, KC_ERR_ARG, "kc_model_generate: bad arguments");
  cudaSetDevice(ctx->device);
  Model& m = *ctx->model;
  if (!m.seq_pos.empty()) m.seq_pos[0] = -1;  // sequence 0 loses its pending token
  if (m.cached + n_prompt + std::max(0, n_gen - 1) > m.n_ctx)
    return fail(ctx, KC_ERR_ARG, "kc_model_generate: context full (n_ctx = %d)", m.n_ctx);
  RC(model_forward(ctx, prompt, false, n_prompt));
  if (n_gen == 0) {
    return check_status(ctx);  // synchronises the stream
  }
  // Decode steps read their token (the previous argmax) and position from
  // device memory and append their argmax to `hist`: no host round trip per
  // token. The first step runs eagerly (it also sizes every buffer for one
  // row); it is then captured once as a CUDA graph and replayed for the rest.
  uint32_t* hist = nullptr;
  CK(cudaMalloc(&hist, (size_t)n_gen * 4));
  int rc = KC_OK;
  const int init[2] = {1, m.cached};
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  auto step = [&]() -> int {
    RC(model_chunk(ctx, m, 1, m.next, true));
    launch_advance(m.next, hist, m.counters, m.counters + 1, ctx->stream);
    CKL();
    return KC_OK;
  };
  if (cudaMemcpyAsync(hist, m.next, 4, cudaMemcpyDeviceToDevice, ctx->stream) != cudaSuccess ||
      cudaMemcpyAsync(m.counters, init, sizeof init, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess)
    rc = fail(ctx, KC_ERR_CUDA, "kc_model_generate: copy failed");
  const bool graphs = ctx->ep.world <= 1 && !ctx->prof.on && ctx->xs.n_layers == 0 && model_graphs_enabled();
  for (int i = 1; i < n_gen && rc == KC_OK; ++i) {
    if (exec) {
      if (cudaGraphLaunch(exec, ctx->stream) != cudaSuccess) rc = fail(ctx, KC_ERR_CUDA, "cudaGraphLaunch failed");
    } else if (i >= 2 && graphs) {
      // Capture on the context's own capture stream, replay on its stream.
      if (!ctx->cap && cudaStreamCreateWithFlags(&ctx->cap, cudaStreamNonBlocking) != cudaSuccess) {
        rc = fail(ctx, KC_ERR_CUDA, "kc_model_generate: capture stream creation failed");
        break;
      }
      cudaStream_t run = ctx->stream;
      if (cudaStreamBeginCapture(ctx->cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        rc = fail(ctx, KC_ERR_CUDA, "kc_model_generate: stream capture failed");
        break;
      }
      ctx->stream = ctx->cap;
      const int src = step();
      ctx->stream = run;
      const cudaError_t ec = cudaStreamEndCapture(ctx->cap, &graph);
      if (src != KC_OK) {
        rc = src;
        break;
      }
      if (ec != cudaSuccess || cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
        rc = fail(ctx, KC_ERR_CUDA, "kc_model_generate: graph capture of a decode step failed");
        break;
      }
      if (cudaGraphLaunch(exec, ctx->stream) != cudaSuccess) rc = fail(ctx, KC_ERR_CUDA, "cudaGraphLaunch failed");
    } else {
      rc = step();
    }
    if (rc == KC_OK) ++m.cached;
  }
  if (rc == KC_OK && cudaMemcpyAsync(out_tokens, hist, (size_t)n_gen * 4, cudaMemcpyDeviceToHost, ctx->stream) !=
                         cudaSuccess)
    rc = fail(ctx, KC_ERR_CUDA, "kc_model_generate: copy failed");
  cudaStreamSynchronize(ctx->stream);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  cudaFree(hist);
  if (rc != KC_OK) return rc;
  return check_status(ctx);
}

// Caches, positions, logits and argmax slots for n_seq sequences (grown, never
// shrunk). Growing the caches drops every cached position.
static int model_sequences(kc_ctx* ctx, Model& m, int n_seq) {
  if (n_seq <= m.n_seq && m.row_pos) return KC_OK;
  CK(cudaStreamSynchronize(ctx->stream));
  const int ns = std::max(n_seq, m.n_seq);
  if (ns > m.n_seq) {
    const size_t bytes = (size_t)ns * m.seq_elems() * 2;
    __half *kc = nullptr, *vc = nullptr;
    if (cudaMalloc(&kc, bytes) != cudaSuccess || cudaMalloc(&vc, bytes) != cudaSuccess) {
      cudaFree(kc);
      cudaFree(vc);
      return fail(ctx, KC_ERR_OOM, "kc_model_set_sequences: KV caches of %d sequences (%.1f GB) do not fit", ns,
                  2.0 * bytes / 1e9);
    }
    CK(cudaMemsetAsync(kc, 0, bytes, ctx->stream));
    CK(cudaMemsetAsync(vc, 0, bytes, ctx->stream));
    cudaFree(m.kc);
    cudaFree(m.vc);
    m.kc = kc;
    m.vc = vc;
    m.cached = 0;
    m.bytes += (int64_t)(ns - m.n_seq) * m.seq_elems() * 4;
  }
  for (void* p : {(void*)m.row_pos, (void*)m.next, (void*)m.logits, (void*)m.rec, (void*)m.seq_tok}) cudaFree(p);
  m.row_pos = nullptr;
  m.next = m.seq_tok = nullptr;
  m.logits = nullptr;
  m.rec = nullptr;
  CK(cudaMalloc(&m.row_pos, (size_t)ns * 4));
  CK(cudaMalloc(&m.next, (size_t)ns * 4));
  CK(cudaMalloc(&m.seq_tok, (size_t)ns * 4));
  CK(cudaMalloc(&m.logits, (size_t)ns * m.n_vocab * 4));
  CK(cudaMalloc(&m.rec, (size_t)std::max(std::min(m.T, 3), ns) * rec_row_bytes(true, std::max(256, m.d))));
  m.n_seq = ns;
  m.seq_pos.assign(ns, -1);
  return KC_OK;
}

int kc_model_set_sequences(kc_ctx* ctx, int n_seq) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!ctx->model) return fail(ctx, KC_ERR_STATE, "kc_model_set_sequences: call kc_model_init first");
  if (n_seq < 1 || n_seq > kMaxSequences)
    return fail(ctx, KC_ERR_ARG, "kc_model_set_sequences: 1 to %d sequences", kMaxSequences);
  cudaSetDevice(ctx->device);
  RC(model_sequences(ctx, *ctx->model, n_seq));
  return KC_OK;
}

// Transformer::forward of a whole prompt in sequence `seq`'s own cache, from
// position 0; the greedy token after it becomes the sequence's pending token.
int kc_model_prefill_seq(kc_ctx* ctx, int seq, const uint32_t* prompt, int n, uint32_t* next_token) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!ctx->model) return fail(ctx, KC_ERR_STATE, "kc_model_prefill_seq: call kc_model_init first");
  if (!prompt || n < 1) return fail(ctx, KC_ERR_ARG, "kc_model_prefill_seq: empty prompt");
  cudaSetDevice(ctx->device);
  Model& m = *ctx->model;
  if (m.seq_pos.empty()) RC(model_sequences(ctx, m, 1));
  if (seq < 0 || seq >= m.n_seq)
    return fail(ctx, KC_ERR_ARG, "kc_model_prefill_seq: sequence %d of %d (kc_model_set_sequences)", seq, m.n_seq);
  const int keep0 = m.cached;  // sequence 0's position (the single-sequence calls' cache)
  m.cur = seq;
  m.cached = 0;
  int rc = model_forward(ctx, prompt, false, n);
  m.cur = 0;
  m.cached = seq == 0 ? (rc == KC_OK ? n : 0) : keep0;
  RC(rc);
  CK(cudaMemcpyAsync(m.seq_tok + seq, m.next, 4, cudaMemcpyDeviceToDevice, ctx->stream));
  if (next_token) CK(cudaMemcpyAsync(next_token, m.next, 4, cudaMemcpyDeviceToHost, ctx->stream));
  RC(check_status(ctx));  // synchronises the stream
  m.seq_pos[seq] = n;
  return KC_OK;
}

// Greedy decode of sequences 0 .. n_seq-1 in lockstep, each from its pending
// token and position. Each step runs one row per sequence, each row computed
// as a batch of one would be (ctx->rows_mode), so each sequence's tokens are
// kc_model_generate's for its prompt alone.
int kc_model_decode_seqs(kc_ctx* ctx, int n_seq, int n_gen, uint32_t* out_tokens) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!ctx->model) return fail(ctx, KC_ERR_STATE, "kc_model_decode_seqs: call kc_model_init first");
  if (n_gen < 0 || (n_gen > 0 && !out_tokens)) return fail(ctx, KC_ERR_ARG, "kc_model_decode_seqs: bad arguments");
  cudaSetDevice(ctx->device);
  Model& m = *ctx->model;
  if (n_seq < 1 || n_seq > m.n_seq || m.seq_pos.empty())
    return fail(ctx, KC_ERR_ARG, "kc_model_decode_seqs: %d sequences of %d", n_seq, m.n_seq);
  for (int s = 0; s < n_seq; ++s) {
    if (m.seq_pos[s] < 1)
      return fail(ctx, KC_ERR_STATE, "kc_model_decode_seqs: sequence %d has no prompt (kc_model_prefill_seq)", s);
    if (m.seq_pos[s] + std::max(0, n_gen - 1) > m.n_ctx)
      return fail(ctx, KC_ERR_ARG, "kc_model_decode_seqs: sequence %d needs more than n_ctx = %d positions", s,
                  m.n_ctx);
  }
  for (auto& kv : ctx->layers)
    if (kv.second.has_router && (int64_t)n_seq * kv.second.k > 1024)
      return fail(ctx, KC_ERR_ARG, "kc_model_decode_seqs: n_seq * top-k must be at most 1024");
  if (n_gen == 0) return KC_OK;
  uint32_t* hist = nullptr;
  CK(cudaMalloc(&hist, (size_t)n_seq * n_gen * 4));
  int rc = KC_OK;
  // Step state: row s reads its token from next[s] (the pending token, then
  // the previous step's argmax) and its position from row_pos[s];
  // advance_rows appends next[s] to sequence s's history (column 0: the
  // pending token).
  const int one = 1;
  if (cudaMemcpy2DAsync(hist, (size_t)n_gen * 4, m.seq_tok, 4, 4, n_seq, cudaMemcpyDeviceToDevice, ctx->stream) !=
          cudaSuccess ||
      cudaMemcpyAsync(m.next, m.seq_tok, (size_t)n_seq * 4, cudaMemcpyDeviceToDevice, ctx->stream) != cudaSuccess ||
      cudaMemcpyAsync(m.row_pos, m.seq_pos.data(), (size_t)n_seq * 4, cudaMemcpyHostToDevice, ctx->stream) !=
          cudaSuccess ||
      cudaMemcpyAsync(m.counters, &one, 4, cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx->stream) != cudaSuccess)
    rc = fail(ctx, KC_ERR_CUDA, "kc_model_decode_seqs: copy failed");
  // The first step runs eagerly (sizing every buffer), the rest replay its
  // CUDA graph.
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  ctx->rows_mode = true;
  auto step = [&]() -> int {
    RC(model_chunk(ctx, m, n_seq, m.next, true, true));
    launch_advance_rows(m.next, hist, n_gen, n_seq, m.counters, m.row_pos, ctx->stream);
    CKL();
    return KC_OK;
  };
  const bool graphs = ctx->ep.world <= 1 && !ctx->prof.on && ctx->xs.n_layers == 0 && model_graphs_enabled();
  for (int i = 1; i < n_gen && rc == KC_OK; ++i) {
    if (exec) {
      if (cudaGraphLaunch(exec, ctx->stream) != cudaSuccess) rc = fail(ctx, KC_ERR_CUDA, "cudaGraphLaunch failed");
    } else if (i >= 2 && graphs) {
      if (!ctx->cap && cudaStreamCreateWithFlags(&ctx->cap, cudaStreamNonBlocking) != cudaSuccess) {
        rc = fail(ctx, KC_ERR_CUDA, "kc_model_decode_seqs: capture stream creation failed");
        break;
      }
      cudaStream_t run = ctx->stream;
      if (cudaStreamBeginCapture(ctx->cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        rc = fail(ctx, KC_ERR_CUDA, "kc_model_decode_seqs: stream capture failed");
        break;
      }
      ctx->stream = ctx->cap;
      const int src = step();
      ctx->stream = run;
      const cudaError_t ec = cudaStreamEndCapture(ctx->cap, &graph);
      if (src != KC_OK) {
        rc = src;
        break;
      }
      if (ec != cudaSuccess || cudaGraphInstantiate(&exec, graph, 0) != cudaSuccess) {
        rc = fail(ctx, KC_ERR_CUDA, "kc_model_decode_seqs: graph capture of a decode step failed");
        break;
      }
      if (cudaGraphLaunch(exec, ctx->stream) != cudaSuccess) rc = fail(ctx, KC_ERR_CUDA, "cudaGraphLaunch failed");
    } else {
      rc = step();
    }
  }
  ctx->rows_mode = false;
  // The last step's argmax (the last token out) is each sequence's new
  // pending token.
  if (rc == KC_OK && n_gen > 1 &&
      cudaMemcpyAsync(m.seq_tok, m.next, (size_t)n_seq * 4, cudaMemcpyDeviceToDevice, ctx->stream) != cudaSuccess)
    rc = fail(ctx, KC_ERR_CUDA, "kc_model_decode_seqs: copy failed");
  if (rc == KC_OK && cudaMemcpyAsync(out_tokens, hist, (size_t)n_seq * n_gen * 4, cudaMemcpyDeviceToHost,
                                     ctx->stream) != cudaSuccess)
    rc = fail(ctx, KC_ERR_CUDA, "kc_model_decode_seqs: copy failed");
  cudaStreamSynchronize(ctx->stream);
  if (exec) cudaGraphExecDestroy(exec);
  if (graph) cudaGraphDestroy(graph);
  cudaFree(hist);
  if (rc != KC_OK) {
    for (int s = 0; s < n_seq; ++s) m.seq_pos[s] = -1;  // partly advanced: needs a new prompt
    m.cached = 0;
    return rc;
  }
  for (int s = 0; s < n_seq; ++s) m.seq_pos[s] += n_gen - 1;
  m.cached = m.seq_pos[0];
  return check_status(ctx);
}

int kc_model_generate_batch(kc_ctx* ctx, int n_seq, const uint32_t* prompts, const int* prompt_lens, int n_gen,
                            uint32_t* out_tokens) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!ctx->model) return fail(ctx, KC_ERR_STATE, "kc_model_generate_batch: call kc_model_init first");
  if (!prompts || !prompt_lens || n_seq < 1 || n_gen < 0 || (n_gen > 0 && !out_tokens))
    return fail(ctx, KC_ERR_ARG, "kc_model_generate_batch: bad arguments");
  if (n_seq > kMaxSequences)
    return fail(ctx, KC_ERR_ARG, "kc_model_generate_batch: at most %d sequences", kMaxSequences);
  cudaSetDevice(ctx->device);
  Model& m = *ctx->model;
  RC(model_finalize(ctx, m));
  for (int s = 0; s < n_seq; ++s) {
    if (prompt_lens[s] < 1) return fail(ctx, KC_ERR_ARG, "kc_model_generate_batch: prompt %d is empty", s);
    if (prompt_lens[s] + std::max(0, n_gen - 1) > m.n_ctx)
      return fail(ctx, KC_ERR_ARG, "kc_model_generate_batch: sequence %d needs more than n_ctx = %d positions", s,
                  m.n_ctx);
  }
  for (auto& kv : ctx->layers)
    if (kv.second.has_router && (int64_t)n_seq * kv.second.k > 1024)
      return fail(ctx, KC_ERR_ARG, "kc_model_generate_batch: n_seq * top-k must be at most 1024");
  RC(model_sequences(ctx, m, n_seq));
  int64_t off = 0;
  for (int s = 0; s < n_seq; ++s) {
    RC(kc_model_prefill_seq(ctx, s, prompts + off, prompt_lens[s], nullptr));
    off += prompt_lens[s];
  }
  return kc_model_decode_seqs(ctx, n_seq, n_gen, out_tokens);
}

int kc_model_truncate(kc_ctx* ctx, int keep) {
  if (!ctx) return KC_ERR_ARG;
  if (!ctx->model) return fail(ctx, KC_ERR_STATE, "kc_model_truncate: no model");
  ctx->model->cached = std::min(ctx->model->cached, std::max(0, keep));
  if (!ctx->model->seq_pos.empty()) ctx->model->seq_pos[0] = -1;
  return KC_OK;
}

int kc_model_cached(const kc_ctx* ctx) { return ctx && ctx->model ? ctx->model->cached : 0; }

// ---- model files -----------------------------------------------------------
int kc_gguf_inspect(const char* path, char* out, int64_t cap) {
  if (!path || (!out && cap > 0)) {
    set_global_error("kc_gguf_inspect: bad arguments");
    return KC_ERR_ARG;
  }
  std::string json, err;
  const int rc = gguf_inspect(path, json, err);
  if (rc != KC_OK) {
    set_global_error(("kc_gguf_inspect: " + err).c_str());
    return rc;
  }
  if ((int64_t)json.size() + 1 > cap) {
    set_global_error("kc_gguf_inspect: output buffer too small");
    return KC_ERR_SHAPE;
  }
  memcpy(out, json.c_str(), json.size() + 1);
  return KC_OK;
}

int kc_load_gguf(kc_ctx* ctx, const char* path, int n_ctx, char* info_json, int64_t cap) {
  if (!ctx) return KC_ERR_ARG;
  ctx->err.clear();
  if (!path || n_ctx < 1) return fail(ctx, KC_ERR_ARG, "kc_load_gguf: bad arguments");
  cudaSetDevice(ctx->device);
  LoadSink s{};
  s.ctx = ctx;
  s.model_init = [](void* c, int nl, int d, int nh, int nkv, int hd, int nv, int nc, int rd, float rb, float eps,
                    int arch) { return kc_model_init((kc_ctx*)c, nl, d, nh, nkv, hd, nv, nc, rd, rb, eps, arch); };
  s.model_tensor = [](void* c, int l, int kind, int t, const void* w, int64_t r, int64_t cl) {
    return kc_model_tensor((kc_ctx*)c, l, kind, t, w, r, cl, 0);
  };
  s.experts = [](void* c, int l, int E, int d, int ff, int tg, const void* g, int tu, const void* u, int td,
                 const void* dn) { return kc_upload_experts((kc_ctx*)c, l, E, d, ff, tg, g, tu, u, td, dn, 0); };
  s.router = [](void* c, int l, const float* w, int E, int d, int k, int nt, float ws) {
    return kc_upload_router((kc_ctx*)c, l, w, E, d, k, nt, ws, 0);
  };
  s.shared = [](void* c, int l, int ff, int d, int tg, const void* g, int tu, const void* u, int td, const void* dn,
                const float* gi) { return kc_upload_shared_expert((kc_ctx*)c, l, ff, d, tg, g, tu, u, td, dn, gi, 0); };
  s.device_bytes_of = [](int t, int64_t rows, int64_t cols) -> int64_t { return dev_matrix_bytes(t, rows, cols); };
  std::string err, info;
  const int rc = gguf_load(path, n_ctx, s, err, info);
  if (info_json && cap > 0) {
    const size_t n = std::min<size_t>(info.size(), (size_t)cap - 1);
    memcpy(info_json, info.data(), n);
    info_json[n] = 0;
  }
  if (rc != KC_OK) {
    if (!err.empty() && ctx->err.empty()) ctx->err = "kc_load_gguf: " + err;
    return rc;
  }
  return KC_OK;
}

}  // extern "C"
