// GGUF / KGUF model loading into the HBM-resident tables (host code).
//
// A reader of the container format that kestrel-gguf parses
// (crates/kestrel-gguf/src/lib.rs:196-311): header, metadata key/values,
// tensor infos, the aligned data section; Kestrel-prepared containers (KGUF
// magic) may stride the outermost slices of a tensor (`kestrel.stride.<name>`
// metadata, TensorInfo::slice_offset, lib.rs:183-189), and the loader reads
// every expert slice at its own offset. Hyper-parameters follow
// kestrel-model's read_hparams and MoeInfo (crates/kestrel-model/src/
// lib.rs:170-215, 338-373); the tensors Transformer::new looks up by name
// (crates/kestrel-engine/src/transformer.rs:147-213) go to kc_model_tensor /
// kc_upload_experts / kc_upload_router / kc_upload_shared_expert.
//
// The placement decision is the VRAM tier the planner lacks (its native_moe
// sizing, crates/kestrel-planner/src/lib.rs:429-439, knows RAM and NVMe): the
// device bytes of every weight in this library's layout, the KV cache and a
// workspace allowance are added up against the GPU's free memory, and a model
// that does not fit is refused before anything is uploaded.
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "loader.h"

namespace {

struct GValue {
  int type = -1;  // GGUF value type
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  bool b = false;
  std::string s;
  std::vector<GValue> arr;
  bool is_int() const { return type <= 5 || type == 10 || type == 11 || type == 7; }
  bool as_u64(uint64_t& out) const {
    if (type == 0 || type == 2 || type == 4 || type == 10) { out = u; return true; }
    if ((type == 1 || type == 3 || type == 5 || type == 11) && i >= 0) { out = (uint64_t)i; return true; }
    return false;
  }
  bool as_f64(double& out) const {
    if (type == 6 || type == 12) { out = f; return true; }
    uint64_t v;
    if (as_u64(v)) { out = (double)v; return true; }
    if (type == 1 || type == 3 || type == 5 || type == 11) { out = (double)i; return true; }
    return false;
  }
};

struct GTensor {
  std::string name;
  std::vector<uint64_t> dims;  // dims[0] is the row length
  int type = 0;
  uint64_t offset = 0, size = 0, stride = 0;  // stride 0: contiguous slices
  uint64_t rows() const {
    uint64_t r = 1;
    for (size_t k = 1; k < dims.size(); ++k) r *= dims[k];
    return r;
  }
  uint64_t n_slices() const { return dims.empty() ? 1 : dims.back(); }
  uint64_t slice_bytes() const { return size / std::max<uint64_t>(1, n_slices()); }
  uint64_t slice_offset(uint64_t s) const { return offset + s * (stride ? stride : slice_bytes()); }
};

// ggml block elements / bytes (crates/kestrel-gguf/src/types.rs:48-191) for
// the types this library has kernels for, plus the common ones a file may
// hold (sizes only, to validate the layout).
bool ggml_block(int t, int& elems, int& bytes) {
  switch (t) {
    case 0: elems = 1; bytes = 4; return true;     // F32
    case 1: elems = 1; bytes = 2; return true;     // F16
    case 2: elems = 32; bytes = 18; return true;   // Q4_0
    case 3: elems = 32; bytes = 20; return true;   // Q4_1
    case 6: elems = 32; bytes = 22; return true;   // Q5_0
    case 7: elems = 32; bytes = 24; return true;   // Q5_1
    case 8: elems = 32; bytes = 34; return true;   // Q8_0
    case 10: elems = 256; bytes = 84; return true; // Q2_K
    case 11: elems = 256; bytes = 110; return true;// Q3_K
    case 12: elems = 256; bytes = 144; return true;// Q4_K
    case 13: elems = 256; bytes = 176; return true;// Q5_K
    case 14: elems = 256; bytes = 210; return true;// Q6_K
    case 30: elems = 1; bytes = 2; return true;    // BF16
    default: return false;
  }
}

struct Gguf {
  std::string err;
  int fd = -1;
  uint64_t file_size = 0, data_offset = 0, alignment = 32;
  uint32_t version = 0;
  bool prepared = false;
  std::map<std::string, GValue> kv;
  std::vector<GTensor> tensors;
  std::map<std::string, size_t> index;
  // buffered sequential reader for the header
  std::vector<uint8_t> buf;
  uint64_t buf_pos = 0, buf_len = 0, pos = 0;

  ~Gguf() {
    if (fd >= 0) close(fd);
  }
  bool fail(const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    if (err.empty()) err = b;
    return false;
  }
  bool read_exact(void* dst, uint64_t n) {
    uint8_t* d = static_cast<uint8_t*>(dst);
    while (n) {
      if (buf_pos == buf_len) {
        if (buf.empty()) buf.resize(1 << 20);
        const ssize_t r = pread(fd, buf.data(), buf.size(), (off_t)pos);
        if (r <= 0) return fail("corrupt GGUF: unexpected end of file at byte %llu", (unsigned long long)pos);
        buf_pos = 0;
        buf_len = (uint64_t)r;
      }
      const uint64_t take = std::min(n, buf_len - buf_pos);
      memcpy(d, buf.data() + buf_pos, take);
      buf_pos += take;
      pos += take;
      d += take;
      n -= take;
    }
    return true;
  }
  template <typename V>
  bool rd(V& v) { return read_exact(&v, sizeof v); }
  bool rd_string(std::string& s) {
    uint64_t n;
    if (!rd(n)) return false;
    if (n > (64ull << 20)) return fail("corrupt GGUF: string of %llu bytes", (unsigned long long)n);
    s.resize(n);
    return n == 0 || read_exact(&s[0], n);
  }
  bool rd_value(int type, GValue& v, int depth = 0) {
    v.type = type;
    switch (type) {
      case 0: { uint8_t x; if (!rd(x)) return false; v.u = x; return true; }
      case 1: { int8_t x; if (!rd(x)) return false; v.i = x; return true; }
      case 2: { uint16_t x; if (!rd(x)) return false; v.u = x; return true; }
      case 3: { int16_t x; if (!rd(x)) return false; v.i = x; return true; }
      case 4: { uint32_t x; if (!rd(x)) return false; v.u = x; return true; }
      case 5: { int32_t x; if (!rd(x)) return false; v.i = x; return true; }
      case 6: { float x; if (!rd(x)) return false; v.f = x; return true; }
      case 7: { uint8_t x; if (!rd(x)) return false; v.b = x != 0; v.u = x; return true; }
      case 8: return rd_string(v.s);
      case 9: {
        if (depth > 2) return fail("corrupt GGUF: nested arrays");
        uint32_t et;
        uint64_t n;
        if (!rd(et) || !rd(n)) return false;
        if (n > (1ull << 28)) return fail("corrupt GGUF: array of %llu elements", (unsigned long long)n);
        v.arr.resize(n);
        for (uint64_t k = 0; k < n; ++k)
          if (!rd_value((int)et, v.arr[k], depth + 1)) return false;
        return true;
      }
      case 10: { uint64_t x; if (!rd(x)) return false; v.u = x; return true; }
      case 11: { int64_t x; if (!rd(x)) return false; v.i = x; return true; }
      case 12: { double x; if (!rd(x)) return false; v.f = x; return true; }
      default: return fail("corrupt GGUF: value type %d", type);
    }
  }

  // GgufFile::open (lib.rs:196-311).
  bool open(const char* path) {
    fd = ::open(path, O_RDONLY);
    if (fd < 0) return fail("cannot open %s", path);
    const off_t end = lseek(fd, 0, SEEK_END);
    if (end < 0) return fail("cannot size %s", path);
    file_size = (uint64_t)end;
    char magic[4];
    if (!read_exact(magic, 4)) return false;
    prepared = memcmp(magic, "KGUF", 4) == 0;
    if (!prepared && memcmp(magic, "GGUF", 4) != 0) return fail("not a GGUF file (bad magic)");
    if (!rd(version)) return false;
    if (version < 2 || version > 3) return fail("unsupported GGUF version %u (supported: 2, 3)", version);
    uint64_t n_tensors, n_kv;
    if (!rd(n_tensors) || !rd(n_kv)) return false;
    if (n_tensors > (1ull << 24) || n_kv > (1ull << 20))
      return fail("corrupt GGUF: implausible counts: %llu tensors, %llu kv", (unsigned long long)n_tensors,
                  (unsigned long long)n_kv);
    for (uint64_t k = 0; k < n_kv; ++k) {
      std::string key;
      uint32_t ty;
      GValue v;
      if (!rd_string(key) || !rd(ty) || !rd_value((int)ty, v)) return false;
      kv[key] = std::move(v);
    }
    auto al = kv.find("general.alignment");
    if (al != kv.end()) {
      uint64_t a;
      if (!al->second.as_u64(a) || a == 0 || (a & (a - 1))) return fail("corrupt GGUF: general.alignment must be a power of two");
      alignment = a;
    }
    tensors.resize(n_tensors);
    std::vector<uint64_t> rel(n_tensors);
    for (uint64_t k = 0; k < n_tensors; ++k) {
      GTensor& t = tensors[k];
      uint32_t nd, ty;
      if (!rd_string(t.name) || !rd(nd)) return false;
      if (nd == 0 || nd > 8) return fail("corrupt GGUF: tensor '%s' has %u dims", t.name.c_str(), nd);
      t.dims.resize(nd);
      for (auto& dd : t.dims)
        if (!rd(dd)) return false;
      if (!rd(ty) || !rd(rel[k])) return false;
      t.type = (int)ty;
    }
    data_offset = (pos + alignment - 1) / alignment * alignment;
    for (uint64_t k = 0; k < n_tensors; ++k) {
      GTensor& t = tensors[k];
      int be, bb;
      if (!ggml_block(t.type, be, bb)) return fail("unknown ggml tensor type id %d for tensor '%s'", t.type, t.name.c_str());
      uint64_t n = 1;
      for (uint64_t dd : t.dims) {
        if (dd && n > UINT64_MAX / dd) return fail("corrupt GGUF: tensor '%s' element count overflows", t.name.c_str());
        n *= dd;
      }
      if (t.dims[0] % (uint64_t)be)
        return fail("corrupt GGUF: tensor '%s': row length %llu not a multiple of block size %d", t.name.c_str(),
                    (unsigned long long)t.dims[0], be);
      t.size = n / be * bb;
      if (rel[k] % alignment) return fail("corrupt GGUF: tensor '%s' offset not aligned", t.name.c_str());
      t.offset = data_offset + rel[k];
      auto st = kv.find("kestrel.stride." + t.name);
      if (st != kv.end()) {
        if (!prepared) return fail("corrupt GGUF: tensor '%s' is strided in a plain GGUF file", t.name.c_str());
        uint64_t s;
        const uint64_t slices = t.n_slices();
        if (!st->second.as_u64(s) || slices < 2 || t.size % slices || s < t.size / slices || s % alignment)
          return fail("corrupt GGUF: tensor '%s': invalid stride", t.name.c_str());
        t.stride = s;
      }
      const uint64_t span = t.stride ? (t.n_slices() - 1) * t.stride + t.slice_bytes() : t.size;
      if (t.offset + span > file_size)
        return fail("corrupt GGUF: tensor '%s' extends past end of file (%llu bytes) -- truncated?", t.name.c_str(),
                    (unsigned long long)file_size);
      index[t.name] = k;
    }
    return true;
  }

  const GTensor* tensor(const std::string& n) const {
    auto it = index.find(n);
    return it == index.end() ? nullptr : &tensors[it->second];
  }
  const GValue* get(const std::string& k) const {
    auto it = kv.find(k);
    return it == kv.end() ? nullptr : &it->second;
  }
  bool get_u64(const std::string& k, uint64_t& v) const {
    const GValue* g = get(k);
    return g && g->as_u64(v);
  }
  bool get_f64(const std::string& k, double& v) const {
    const GValue* g = get(k);
    return g && g->as_f64(v);
  }
  // scalar_or_max (kestrel-model lib.rs:375-381)
  bool get_u64_or_max(const std::string& k, uint64_t& v) const {
    const GValue* g = get(k);
    if (!g) return false;
    if (g->type == 9) {
      bool any = false;
      v = 0;
      for (const auto& e : g->arr) {
        uint64_t x;
        if (e.as_u64(x)) { v = std::max(v, x); any = true; }
      }
      return any;
    }
    return g->as_u64(v);
  }
  // Bytes [off, off + n) of the file into dst.
  bool read_at(uint64_t off, void* dst, uint64_t n) {
    uint8_t* d = static_cast<uint8_t*>(dst);
    while (n) {
      const ssize_t r = pread(fd, d, std::min<uint64_t>(n, 1ull << 30), (off_t)off);
      if (r <= 0) return fail("read of %llu bytes at %llu failed", (unsigned long long)n, (unsigned long long)off);
      d += r;
      off += (uint64_t)r;
      n -= (uint64_t)r;
    }
    return true;
  }
  // The whole tensor, slices gathered in order (strided or not).
  bool read_tensor(const GTensor& t, std::vector<uint8_t>& out) {
    out.resize(t.size);
    if (!t.stride) return read_at(t.offset, out.data(), t.size);
    const uint64_t sb = t.slice_bytes();
    for (uint64_t s = 0; s < t.n_slices(); ++s)
      if (!read_at(t.slice_offset(s), out.data() + s * sb, sb)) return false;
    return true;
  }
};

// Hyper-parameters and MoE options (kestrel-model read_hparams / MoeInfo).
struct ModelDesc {
  std::string arch;
  int kc_arch = KC_ARCH_QWEN3;
  uint64_t n_layer = 0, n_embd = 0, n_head = 0, n_head_kv = 0, head_dim = 0, n_vocab = 0, rope_dim = 0;
  double rope_base = 10000.0, eps = 1e-5;
  uint64_t n_expert = 0, n_expert_used = 0, n_ff_exp = 0, n_ff_shexp = 0;
  bool norm_topk = true;
  double weights_scale = 0.0;
};

bool describe(const Gguf& g, ModelDesc& m, std::string& err) {
  const GValue* a = g.get("general.architecture");
  if (!a || a->type != 8) { err = "general.architecture missing"; return false; }
  m.arch = a->s;
  if (m.arch == "llama") m.kc_arch = KC_ARCH_LLAMA;
  else if (m.arch == "qwen2" || m.arch == "qwen2moe") m.kc_arch = KC_ARCH_QWEN2;
  else if (m.arch == "qwen3" || m.arch == "qwen3moe") m.kc_arch = KC_ARCH_QWEN3;
  else { err = "architecture '" + m.arch + "' (native: llama, qwen2, qwen3, qwen2moe, qwen3moe)"; return false; }
  const std::string p = m.arch + ".";
  if (!g.get_u64(p + "block_count", m.n_layer) || !g.get_u64(p + "embedding_length", m.n_embd) ||
      !g.get_u64_or_max(p + "attention.head_count", m.n_head)) {
    err = "missing " + p + "block_count / embedding_length / attention.head_count";
    return false;
  }
  if (!g.get_u64_or_max(p + "attention.head_count_kv", m.n_head_kv)) m.n_head_kv = m.n_head;
  const GValue* hkv = g.get(p + "attention.head_count_kv");
  if (hkv && hkv->type == 9)
    for (const auto& e : hkv->arr) {
      uint64_t x;
      if (e.as_u64(x) && x != m.n_head_kv) { err = "per-layer KV head counts"; return false; }
    }
  m.head_dim = m.n_head ? m.n_embd / m.n_head : 0;
  uint64_t hk = 0, hv = 0;
  if (g.get_u64(p + "attention.key_length", hk)) m.head_dim = hk;
  if (g.get_u64(p + "attention.value_length", hv) && hv != m.head_dim) { err = "key/value head sizes differ"; return false; }
  if (!g.get_u64(p + "vocab_size", m.n_vocab)) {
    const GTensor* e = g.tensor("token_embd.weight");
    m.n_vocab = e && e->dims.size() > 1 ? e->dims[1] : 0;
  }
  if (!g.get_f64(p + "rope.freq_base", m.rope_base)) m.rope_base = 10000.0;
  if (!g.get_u64(p + "rope.dimension_count", m.rope_dim)) m.rope_dim = m.head_dim;
  if (!g.get_f64(p + "attention.layer_norm_rms_epsilon", m.eps)) m.eps = 1e-5;
  g.get_u64(p + "expert_count", m.n_expert);
  g.get_u64(p + "expert_used_count", m.n_expert_used);
  if (!g.get_u64(p + "expert_feed_forward_length", m.n_ff_exp)) {
    const GTensor* t = g.tensor("blk.0.ffn_gate_exps.weight");
    m.n_ff_exp = t && t->dims.size() > 1 ? t->dims[1] : 0;
  }
  g.get_u64(p + "expert_shared_feed_forward_length", m.n_ff_shexp);
  const GValue* nt = g.get(p + "expert_weights_norm");
  m.norm_topk = nt && nt->type == 7 ? nt->b : m.arch != "qwen2moe";
  if (!g.get_f64(p + "expert_weights_scale", m.weights_scale)) m.weights_scale = 0.0;
  if (m.n_layer == 0 || m.n_embd == 0 || m.n_head == 0 || m.n_vocab == 0) { err = "empty hyper-parameters"; return false; }
  return true;
}

std::string json_escape(const std::string& s) {
  std::string o;
  for (char c : s) {
    if (c == '"' || c == '\\') { o += '\\'; o += c; }
    else if ((unsigned char)c < 0x20) { char b[8]; snprintf(b, sizeof b, "\\u%04x", c); o += b; }
    else o += c;
  }
  return o;
}

}  // namespace

namespace kc {

// Parse `path` and describe it as JSON (no GPU needed).
int gguf_inspect(const char* path, std::string& json, std::string& err) {
  Gguf g;
  if (!g.open(path)) { err = g.err; return KC_ERR_ARG; }
  ModelDesc m;
  std::string derr;
  const bool ok = describe(g, m, derr);
  char b[1024];
  snprintf(b, sizeof b,
           "{\"version\": %u, \"prepared\": %s, \"alignment\": %llu, \"data_offset\": %llu, \"n_tensors\": %zu, "
           "\"n_kv\": %zu",
           g.version, g.prepared ? "true" : "false", (unsigned long long)g.alignment,
           (unsigned long long)g.data_offset, g.tensors.size(), g.kv.size());
  json = b;
  if (ok) {
    snprintf(b, sizeof b,
             ", \"arch\": \"%s\", \"n_layer\": %llu, \"n_embd\": %llu, \"n_head\": %llu, \"n_head_kv\": %llu, "
             "\"head_dim\": %llu, \"n_vocab\": %llu, \"rope_dim\": %llu, \"rope_base\": %.9g, \"rms_eps\": %.9g, "
             "\"n_expert\": %llu, \"n_expert_used\": %llu, \"n_ff_exp\": %llu, \"norm_topk\": %s, "
             "\"weights_scale\": %.9g",
             json_escape(m.arch).c_str(), (unsigned long long)m.n_layer, (unsigned long long)m.n_embd,
             (unsigned long long)m.n_head, (unsigned long long)m.n_head_kv, (unsigned long long)m.head_dim,
             (unsigned long long)m.n_vocab, (unsigned long long)m.rope_dim, m.rope_base, m.eps,
             (unsigned long long)m.n_expert, (unsigned long long)m.n_expert_used, (unsigned long long)m.n_ff_exp,
             m.norm_topk ? "true" : "false", m.weights_scale);
    json += b;
  } else {
    json += ", \"model_error\": \"" + json_escape(derr) + "\"";
  }
  json += ", \"tensors\": [";
  for (size_t k = 0; k < g.tensors.size(); ++k) {
    const GTensor& t = g.tensors[k];
    json += k ? ", " : "";
    json += "{\"name\": \"" + json_escape(t.name) + "\", \"type\": " + std::to_string(t.type) + ", \"dims\": [";
    for (size_t d = 0; d < t.dims.size(); ++d) json += (d ? ", " : "") + std::to_string(t.dims[d]);
    json += "], \"offset\": " + std::to_string(t.offset) + ", \"size\": " + std::to_string(t.size) +
            ", \"stride\": " + std::to_string(t.stride) + "}";
  }
  json += "]}";
  return KC_OK;
}

int gguf_load(const char* path, int n_ctx, const LoadSink& sink, std::string& err, std::string& info) {
  Gguf g;
  if (!g.open(path)) { err = g.err; return KC_ERR_ARG; }
  ModelDesc m;
  if (!describe(g, m, err)) return KC_ERR_ARG;
  auto T = [&](const std::string& n) { return g.tensor(n); };
  auto supported = [](int t) { return t == T_F32 || t == T_Q8_0 || t == T_Q4_K || t == T_Q6_K; };
  // Check every tensor the forward pass reads and add up its device bytes.
  int64_t need = 0;
  std::vector<const GTensor*> uses;
  auto use = [&](const GTensor* t, bool required, const std::string& n) -> int {
    if (!t) {
      if (required) { err = "missing tensor " + n; return KC_ERR_ARG; }
      return KC_OK;
    }
    if (!supported(t->type)) {
      err = "tensor " + n + " has ggml type " + std::to_string(t->type) + " (kernels: F32 Q8_0 Q4_K Q6_K)";
      return KC_ERR_TYPE;
    }
    need += sink.device_bytes_of(t->type, (int64_t)t->rows(), (int64_t)t->dims[0]);
    uses.push_back(t);
    return KC_OK;
  };
  int rc;
  if ((rc = use(T("token_embd.weight"), true, "token_embd.weight"))) return rc;
  if ((rc = use(T("output_norm.weight"), true, "output_norm.weight"))) return rc;
  if ((rc = use(T("output.weight"), false, "output.weight"))) return rc;
  if (!T("output.weight")) need += sink.device_bytes_of(T("token_embd.weight")->type, (int64_t)m.n_vocab, (int64_t)m.n_embd);
  const char* layer_names[] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q.bias", "attn_k.bias",
                               "attn_v.bias", "attn_q_norm", "attn_k_norm", "ffn_norm", "ffn_gate", "ffn_up",
                               "ffn_down", "ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps",
                               "ffn_gate_shexp", "ffn_up_shexp", "ffn_down_shexp", "ffn_gate_inp_shexp"};
  for (uint64_t l = 0; l < m.n_layer; ++l)
    for (const char* nm : layer_names) {
      std::string n = "blk." + std::to_string(l) + "." + nm;
      if (n.find(".bias") == std::string::npos) n += ".weight";
      const bool req = !strcmp(nm, "attn_norm") || !strcmp(nm, "attn_q") || !strcmp(nm, "attn_k") ||
                       !strcmp(nm, "attn_v") || !strcmp(nm, "attn_output") || !strcmp(nm, "ffn_norm");
      if ((rc = use(T(n), req, n))) return rc;
    }
  const int64_t kv_bytes = 2 * (int64_t)m.n_layer * n_ctx * (int64_t)(m.n_head_kv * m.head_dim) * 2;
  const int64_t work = 512ll << 20;  // workspace and activation allowance
  size_t free_b = 0, total_b = 0;
  if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) { err = "cudaMemGetInfo failed"; return KC_ERR_CUDA; }
  const int64_t total_need = need + kv_bytes + work;
  char b[512];
  snprintf(b, sizeof b, "{\"arch\": \"%s\", \"weights_bytes\": %lld, \"kv_bytes\": %lld, \"free_bytes\": %lld, "
           "\"n_layer\": %llu, \"n_vocab\": %llu, \"n_expert\": %llu}", json_escape(m.arch).c_str(),
           (long long)need, (long long)kv_bytes, (long long)free_b, (unsigned long long)m.n_layer,
           (unsigned long long)m.n_vocab, (unsigned long long)m.n_expert);
  info = b;
  if ((int64_t)free_b < total_need) {
    snprintf(b, sizeof b, "model needs %.2f GB of HBM (weights %.2f, KV cache %.2f) but %.2f GB are free; "
             "host-streamed experts are not supported", total_need / 1e9, need / 1e9, kv_bytes / 1e9, free_b / 1e9);
    err = b;
    return KC_ERR_OOM;
  }
  if ((rc = sink.model_init(sink.ctx, (int)m.n_layer, (int)m.n_embd, (int)m.n_head, (int)m.n_head_kv,
                            (int)m.head_dim, (int)m.n_vocab, n_ctx, (int)m.rope_dim, (float)m.rope_base,
                            (float)m.eps, m.kc_arch)))
    return rc;
  std::vector<uint8_t> data;
  auto put = [&](int layer, int kind, const GTensor* t) -> int {
    if (!t) return KC_OK;
    if (!g.read_tensor(*t, data)) { err = g.err; return KC_ERR_ARG; }
    return sink.model_tensor(sink.ctx, layer, kind, t->type, data.data(), (int64_t)t->rows(), (int64_t)t->dims[0]);
  };
  if ((rc = put(-1, KC_T_TOKEN_EMBD, T("token_embd.weight")))) return rc;
  if ((rc = put(-1, KC_T_OUTPUT_NORM, T("output_norm.weight")))) return rc;
  if ((rc = put(-1, KC_T_OUTPUT, T("output.weight")))) return rc;
  for (uint64_t l = 0; l < m.n_layer; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    const struct { const char* n; int kind; } dense[] = {
        {"attn_norm.weight", KC_T_ATTN_NORM}, {"attn_q.weight", KC_T_ATTN_Q}, {"attn_k.weight", KC_T_ATTN_K},
        {"attn_v.weight", KC_T_ATTN_V}, {"attn_output.weight", KC_T_ATTN_OUT}, {"attn_q.bias", KC_T_ATTN_Q_BIAS},
        {"attn_k.bias", KC_T_ATTN_K_BIAS}, {"attn_v.bias", KC_T_ATTN_V_BIAS}, {"attn_q_norm.weight", KC_T_ATTN_Q_NORM},
        {"attn_k_norm.weight", KC_T_ATTN_K_NORM}, {"ffn_norm.weight", KC_T_FFN_NORM}, {"ffn_gate.weight", KC_T_FFN_GATE},
        {"ffn_up.weight", KC_T_FFN_UP}, {"ffn_down.weight", KC_T_FFN_DOWN}};
    for (const auto& dn : dense)
      if ((rc = put((int)l, dn.kind, T(p + dn.n)))) return rc;
    const GTensor *gi = T(p + "ffn_gate_inp.weight"), *ge = T(p + "ffn_gate_exps.weight"),
                  *ue = T(p + "ffn_up_exps.weight"), *de = T(p + "ffn_down_exps.weight");
    if (gi && ge && ue && de) {
      const uint64_t E = ge->n_slices(), ff = ge->dims.size() > 1 ? ge->dims[1] : 0;
      if (E != m.n_expert || gi->type != T_F32 || gi->rows() != E || gi->dims[0] != m.n_embd) {
        err = p + "ffn_gate_inp / *_exps shapes do not match expert_count";
        return KC_ERR_SHAPE;
      }
      std::vector<uint8_t> gd, ud, dd;
      if (!g.read_tensor(*ge, gd) || !g.read_tensor(*ue, ud) || !g.read_tensor(*de, dd)) { err = g.err; return KC_ERR_ARG; }
      if ((rc = sink.experts(sink.ctx, (int)l, (int)E, (int)m.n_embd, (int)ff, ge->type, gd.data(), ue->type,
                             ud.data(), de->type, dd.data())))
        return rc;
      if (!g.read_tensor(*gi, data)) { err = g.err; return KC_ERR_ARG; }
      if ((rc = sink.router(sink.ctx, (int)l, reinterpret_cast<const float*>(data.data()), (int)E, (int)m.n_embd,
                            (int)std::max<uint64_t>(1, m.n_expert_used), m.norm_topk ? 1 : 0, (float)m.weights_scale)))
        return rc;
      const GTensor *sg = T(p + "ffn_gate_shexp.weight"), *su = T(p + "ffn_up_shexp.weight"),
                    *sd = T(p + "ffn_down_shexp.weight"), *si = T(p + "ffn_gate_inp_shexp.weight");
      if (sg && su && sd) {
        std::vector<uint8_t> sgd, sud, sdd, sid;
        if (!g.read_tensor(*sg, sgd) || !g.read_tensor(*su, sud) || !g.read_tensor(*sd, sdd) ||
            (si && !g.read_tensor(*si, sid))) { err = g.err; return KC_ERR_ARG; }
        if (si && si->type != T_F32) { err = p + "ffn_gate_inp_shexp is not F32"; return KC_ERR_TYPE; }
        if ((rc = sink.shared(sink.ctx, (int)l, (int)sg->rows(), (int)m.n_embd, sg->type, sgd.data(), su->type,
                              sud.data(), sd->type, sdd.data(),
                              si ? reinterpret_cast<const float*>(sid.data()) : nullptr)))
          return rc;
      }
    }
  }
  return KC_OK;
}

}  // namespace kc
