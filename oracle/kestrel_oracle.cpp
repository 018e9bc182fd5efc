// TEST INFRASTRUCTURE ONLY -- never linked into, loaded by, or called from the
// product path (kestrel_b200/). Only tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference legs of bench.py load this library, and only
// as the checker or the timed CPU baseline.
//
// A C++17 restatement of the CPU arithmetic of Kestrel's native executor on
// the Mixture-of-Experts FFN path (Eduardo7125/kestrel, crates/kestrel-engine).
// The reference is Rust and cannot be compiled in this image (no cargo/rustc),
// so this file re-states its algorithms with the same floating-point operation
// order, the same x86 SIMD lane structure (AVX2 + FMA + F16C) and the same
// dispatch rules. Build flags: -O2 -mavx2 -mfma -mf16c -ffp-contract=off
// (Rust never contracts a*b+c into an FMA; only explicit _mm256_fmadd_ps is
// fused). Every function cites the reference lines it follows.
//
// Besides the AVX2 kernels (the timed "reference CPU path"), the file holds
// scalar *lane emulations* of the same kernels: plain C loops that compute the
// eight 32-bit lanes explicitly. Tests require the two to agree bit for bit;
// the lane emulations are the specification the CUDA kernels reproduce.

#include <immintrin.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// ggml type ids (crates/kestrel-gguf/src/types.rs:48-86).
enum GgmlType : int {
  T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7,
  T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_BF16 = 30,
};

// Block elements / bytes (types.rs:120-182).
int blk_elems(int t) {
  switch (t) {
    case T_F32: case T_F16: case T_BF16: return 1;
    case T_Q4_0: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_Q8_0: return 32;
    case T_Q4_K: case T_Q5_K: case T_Q6_K: return 256;
    default: return 0;
  }
}
int blk_bytes(int t) {
  switch (t) {
    case T_F32: return 4;
    case T_F16: case T_BF16: return 2;
    case T_Q4_0: return 18;
    case T_Q4_1: return 20;
    case T_Q5_0: return 22;
    case T_Q5_1: return 24;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    default: return 0;
  }
}
// GgmlType::bytes_for (types.rs:185-191): None unless n is a block multiple.
int64_t bytes_for(int t, int64_t n) {
  int be = blk_elems(t);
  if (be == 0 || n % be) return -1;
  return n / be * blk_bytes(t);
}

// Exact f16 -> f32 (quant.rs:13-22 uses the `half` crate LUT; F16C is exact).
inline float h2f(const uint8_t* p) {
  uint16_t h = (uint16_t)(p[0] | (p[1] << 8));
  return _cvtsh_ss(h);
}

// ---------------------------------------------------------------------------
// Thread pool: tiles of output rows are independent (each output element is
// written by exactly one tile), so threading never changes results
// (quant.rs:244-257, 264-278 run the same tiles on rayon). Like rayon's pool
// the workers persist between parallel regions (a region costs a wake-up,
// not thread creation), so the timed CPU baseline is not dominated by
// spawning threads for each of a layer's small products.
int g_threads = 1;

class Pool {
 public:
  ~Pool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  // Runs fn(0..n-1) on the caller and nt - 1 workers (one region at a time).
  void run(int nt, int64_t n, const std::function<void(int64_t)>& fn) {
    std::lock_guard<std::mutex> region(run_mu_);
    while ((int)workers_.size() < nt - 1) {
      const int idx = (int)workers_.size();
      workers_.emplace_back([this, idx] { loop(idx); });
    }
    {
      std::lock_guard<std::mutex> lk(mu_);
      fn_ = &fn;
      n_ = n;
      next_.store(0);
      want_ = nt - 1;
      pending_ = nt - 1;
      ++gen_;
    }
    cv_.notify_all();
    for (int64_t i; (i = next_.fetch_add(1)) < n;) fn(i);
    std::unique_lock<std::mutex> lk(mu_);
    done_.wait(lk, [&] { return pending_ == 0; });
  }

 private:
  void loop(int idx) {
    uint64_t seen = 0;
    std::unique_lock<std::mutex> lk(mu_);
    for (;;) {
      cv_.wait(lk, [&] { return stop_ || gen_ != seen; });
      if (stop_) return;
      seen = gen_;
      if (idx >= want_) continue;
      const std::function<void(int64_t)>* fn = fn_;
      const int64_t n = n_;
      lk.unlock();
      for (int64_t i; (i = next_.fetch_add(1)) < n;) (*fn)(i);
      lk.lock();
      if (--pending_ == 0) done_.notify_one();
    }
  }
  std::mutex run_mu_, mu_;
  std::condition_variable cv_, done_;
  std::vector<std::thread> workers_;
  const std::function<void(int64_t)>* fn_ = nullptr;
  int64_t n_ = 0;
  std::atomic<int64_t> next_{0};
  int want_ = 0, pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

void parallel_for(int64_t n, const std::function<void(int64_t)>& fn) {
  int nt = (int)std::min<int64_t>(g_threads, n);
  if (nt <= 1) {
    for (int64_t i = 0; i < n; ++i) fn(i);
    return;
  }
  static Pool pool;
  pool.run(nt, n, fn);
}

// scale_min_k4 (quant.rs:54-60, qdot.rs:66-72, avx2.rs:78-84).
inline void scale_min_k4(int j, const uint8_t* q, int* sc, int* m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// ---------------------------------------------------------------------------
// dequant_row (quant.rs:63-205). Separate multiplies and subtractions, in the
// order the Rust expressions evaluate them.
void dequant_row(int t, const uint8_t* src, int64_t n, float* y) {
  switch (t) {
    case T_F32:
      std::memcpy(y, src, n * 4);
      return;
    case T_F16:
      for (int64_t i = 0; i < n; ++i) y[i] = h2f(src + 2 * i);
      return;
    case T_BF16:
      for (int64_t i = 0; i < n; ++i) {
        uint32_t b = (uint32_t)(src[2 * i] | (src[2 * i + 1] << 8)) << 16;
        std::memcpy(&y[i], &b, 4);
      }
      return;
    case T_Q8_0:
      for (int64_t b = 0; b < n / 32; ++b) {
        const uint8_t* blk = src + b * 34;
        float d = h2f(blk);
        for (int j = 0; j < 32; ++j) y[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
      }
      return;
    case T_Q4_0:
      for (int64_t b = 0; b < n / 32; ++b) {
        const uint8_t* blk = src + b * 18;
        float d = h2f(blk);
        for (int j = 0; j < 16; ++j) {
          y[b * 32 + j] = (float)((blk[2 + j] & 0xF) - 8) * d;
          y[b * 32 + j + 16] = (float)((blk[2 + j] >> 4) - 8) * d;
        }
      }
      return;
    case T_Q4_1:
      for (int64_t b = 0; b < n / 32; ++b) {
        const uint8_t* blk = src + b * 20;
        float d = h2f(blk), m = h2f(blk + 2);
        for (int j = 0; j < 16; ++j) {
          y[b * 32 + j] = (float)(blk[4 + j] & 0xF) * d + m;
          y[b * 32 + j + 16] = (float)(blk[4 + j] >> 4) * d + m;
        }
      }
      return;
    case T_Q5_0:
    case T_Q5_1: {
      bool one = t == T_Q5_1;
      int bs = one ? 24 : 22, off = one ? 4 : 2;
      for (int64_t b = 0; b < n / 32; ++b) {
        const uint8_t* blk = src + b * bs;
        float d = h2f(blk), m = one ? h2f(blk + 2) : 0.f;
        uint32_t qh;
        std::memcpy(&qh, blk + off, 4);
        const uint8_t* qs = blk + off + 4;
        for (int j = 0; j < 16; ++j) {
          uint8_t h0 = (uint8_t)(((qh >> j) << 4) & 0x10);
          uint8_t h1 = (uint8_t)((qh >> (j + 12)) & 0x10);
          int v0 = (qs[j] & 0xF) | h0, v1 = (qs[j] >> 4) | h1;
          if (one) {
            y[b * 32 + j] = (float)v0 * d + m;
            y[b * 32 + j + 16] = (float)v1 * d + m;
          } else {
            y[b * 32 + j] = (float)(v0 - 16) * d;
            y[b * 32 + j + 16] = (float)(v1 - 16) * d;
          }
        }
      }
      return;
    }
    case T_Q4_K:
      for (int64_t b = 0; b < n / 256; ++b) {
        const uint8_t* blk = src + b * 144;
        float d = h2f(blk), dmin = h2f(blk + 2);
        const uint8_t* sc = blk + 4;
        const uint8_t* qs = blk + 16;
        for (int k = 0; k < 4; ++k) {
          int s1, m1, s2, m2;
          scale_min_k4(2 * k, sc, &s1, &m1);
          scale_min_k4(2 * k + 1, sc, &s2, &m2);
          float d1 = d * (float)s1, mm1 = dmin * (float)m1;
          float d2 = d * (float)s2, mm2 = dmin * (float)m2;
          float* yy = y + b * 256 + k * 64;
          for (int l = 0; l < 32; ++l) {
            yy[l] = d1 * (float)(qs[32 * k + l] & 0xF) - mm1;
            yy[l + 32] = d2 * (float)(qs[32 * k + l] >> 4) - mm2;
          }
        }
      }
      return;
    case T_Q5_K:
      for (int64_t b = 0; b < n / 256; ++b) {
        const uint8_t* blk = src + b * 176;
        float d = h2f(blk), dmin = h2f(blk + 2);
        const uint8_t* sc = blk + 4;
        const uint8_t* qh = blk + 16;
        const uint8_t* ql = blk + 48;
        uint8_t u1 = 1, u2 = 2;
        for (int k = 0; k < 4; ++k) {
          int s1, m1, s2, m2;
          scale_min_k4(2 * k, sc, &s1, &m1);
          scale_min_k4(2 * k + 1, sc, &s2, &m2);
          float d1 = d * (float)s1, mm1 = dmin * (float)m1;
          float d2 = d * (float)s2, mm2 = dmin * (float)m2;
          float* yy = y + b * 256 + k * 64;
          for (int l = 0; l < 32; ++l) {
            int hi1 = (qh[l] & u1) ? 16 : 0, hi2 = (qh[l] & u2) ? 16 : 0;
            yy[l] = d1 * (float)((ql[32 * k + l] & 0xF) + hi1) - mm1;
            yy[l + 32] = d2 * (float)((ql[32 * k + l] >> 4) + hi2) - mm2;
          }
          u1 <<= 2;
          u2 <<= 2;
        }
      }
      return;
    case T_Q6_K:
      for (int64_t b = 0; b < n / 256; ++b) {
        const uint8_t* blk = src + b * 210;
        float d = h2f(blk + 208);
        for (int h = 0; h < 2; ++h) {
          const uint8_t* ql = blk + h * 64;
          const uint8_t* qh = blk + 128 + h * 32;
          const int8_t* sc = (const int8_t*)(blk + 192 + h * 8);
          float* yy = y + b * 256 + h * 128;
          for (int l = 0; l < 32; ++l) {
            int is = l / 16;
            int q1 = ((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
            int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
            int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
            int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            yy[l] = d * (float)sc[is] * (float)q1;
            yy[l + 32] = d * (float)sc[is + 2] * (float)q2;
            yy[l + 64] = d * (float)sc[is + 4] * (float)q3;
            yy[l + 96] = d * (float)sc[is + 6] * (float)q4;
          }
        }
      }
      return;
    default:
      return;
  }
}

// quant::dot (quant.rs:208-224): eight accumulators, separate mul and add,
// `acc.iter().sum()` (a sequential fold that starts at -0.0), then the tail.
float dot_scalar(const float* a, const float* b, int64_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int64_t n8 = n / 8 * 8;
  for (int64_t c = 0; c < n8; c += 8)
    for (int i = 0; i < 8; ++i) acc[i] = acc[i] + a[c + i] * b[c + i];
  float s = -0.0f;
  for (int i = 0; i < 8; ++i) s = s + acc[i];
  for (int64_t c = n8; c < n; ++c) s = s + a[c] * b[c];
  return s;
}

// ---------------------------------------------------------------------------
// Activation quantization.
// Rust `(v).round() as i32` is round-half-away-from-zero with a saturating,
// NaN->0 cast; `.clamp(-127, 127)` follows.
inline int8_t q8_round(float v) {
  float r = std::round(v);
  int32_t i;
  if (std::isnan(r)) i = 0;
  else if (r >= 2147483647.f) i = INT32_MAX;
  else if (r <= -2147483648.f) i = INT32_MIN;
  else i = (int32_t)r;
  return (int8_t)std::min(127, std::max(-127, i));
}

// Q8Row::quantize (qdot.rs:29-49): blocks of 32, Σq per 16.
void q8_quantize(const float* x, int64_t n, int8_t* q, float* d, int32_t* s16) {
  for (int64_t b = 0; b < n / 32; ++b) {
    const float* xs = x + b * 32;
    float amax = 0.f;
    for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(xs[j]));
    float scale = amax / 127.0f;
    float inv = scale > 0.f ? 1.0f / scale : 0.f;
    d[b] = scale;
    for (int j = 0; j < 32; ++j) q[b * 32 + j] = q8_round(xs[j] * inv);
    int32_t s0 = 0, s1 = 0;
    for (int j = 0; j < 16; ++j) s0 += q[b * 32 + j];
    for (int j = 16; j < 32; ++j) s1 += q[b * 32 + j];
    s16[2 * b] = s0;
    s16[2 * b + 1] = s1;
  }
}

// Q8KRow::quantize (qdot.rs:347-367): blocks of 256, Σq per 16 (bsums).
// Kestrel's own definition (d = amax/127), not ggml's quantize_row_q8_K.
void q8k_quantize(const float* x, int64_t n, int8_t* q, float* d, int32_t* bsums) {
  for (int64_t b = 0; b < n / 256; ++b) {
    const float* xs = x + b * 256;
    float amax = 0.f;
    for (int j = 0; j < 256; ++j) amax = std::fmax(amax, std::fabs(xs[j]));
    float scale = amax / 127.0f;
    float inv = scale > 0.f ? 1.0f / scale : 0.f;
    d[b] = scale;
    for (int j = 0; j < 256; ++j) q[b * 256 + j] = q8_round(xs[j] * inv);
  }
  for (int64_t k = 0; k < n / 16; ++k) {
    int32_t s = 0;
    for (int j = 0; j < 16; ++j) s += q[k * 16 + j];
    bsums[k] = s;
  }
}

// ---------------------------------------------------------------------------
// AVX2 helpers (avx2.rs:19-46).
inline float hsum(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v);
  __m128 hi = _mm256_extractf128_ps(v, 1);
  __m128 s = _mm_add_ps(lo, hi);
  s = _mm_add_ps(s, _mm_movehl_ps(s, s));
  s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 1));
  return _mm_cvtss_f32(s);
}
// Scalar statement of hsum's addition tree.
inline float hsum8(const float* v) {
  return ((v[0] + v[4]) + (v[2] + v[6])) + ((v[1] + v[5]) + (v[3] + v[7]));
}
inline __m256i ld(const void* p) { return _mm256_loadu_si256((const __m256i*)p); }
inline __m256i madd_u8i8(__m256i w, __m256i x) {
  return _mm256_madd_epi16(_mm256_maddubs_epi16(w, x), _mm256_set1_epi16(1));
}
inline __m256i madd_i8i8(__m256i w, __m256i x) {
  return madd_u8i8(_mm256_sign_epi8(w, w), _mm256_sign_epi8(x, w));
}

// Q8Row dots (avx2.rs:48-147).
float dot_q8_0(const uint8_t* w, int64_t n, const int8_t* q, const float* d) {
  __m256 acc = _mm256_setzero_ps();
  for (int64_t b = 0; b < n / 32; ++b) {
    const uint8_t* blk = w + b * 34;
    __m256 p = _mm256_cvtepi32_ps(madd_i8i8(ld(blk + 2), ld(q + b * 32)));
    acc = _mm256_fmadd_ps(p, _mm256_set1_ps(h2f(blk) * d[b]), acc);
  }
  return hsum(acc);
}

float dot_q4_0(const uint8_t* w, int64_t n, const int8_t* q, const float* d) {
  __m256 acc = _mm256_setzero_ps();
  const __m256i m4 = _mm256_set1_epi8(0x0F), eight = _mm256_set1_epi8(8);
  for (int64_t b = 0; b < n / 32; ++b) {
    const uint8_t* blk = w + b * 18;
    __m128i v = _mm_loadu_si128((const __m128i*)(blk + 2));
    __m256i both = _mm256_set_m128i(_mm_srli_epi16(v, 4), v);
    __m256i qw = _mm256_sub_epi8(_mm256_and_si256(both, m4), eight);
    __m256 p = _mm256_cvtepi32_ps(madd_i8i8(qw, ld(q + b * 32)));
    acc = _mm256_fmadd_ps(p, _mm256_set1_ps(h2f(blk) * d[b]), acc);
  }
  return hsum(acc);
}

float dot_q4_k_q8(const uint8_t* w, int64_t n, const int8_t* q, const float* d, const int32_t* s16) {
  __m256 acc = _mm256_setzero_ps();
  float mins = 0.f;
  const __m256i m4 = _mm256_set1_epi8(0x0F);
  for (int64_t sb = 0; sb < n / 256; ++sb) {
    const uint8_t* blk = w + sb * 144;
    float dd = h2f(blk), dmin = h2f(blk + 2);
    const uint8_t* sc = blk + 4;
    for (int k = 0; k < 4; ++k) {
      __m256i v = ld(blk + 16 + 32 * k);
      __m256i lo = _mm256_and_si256(v, m4);
      __m256i hi = _mm256_and_si256(_mm256_srli_epi16(v, 4), m4);
      int64_t b0 = sb * 8 + 2 * k, b1 = b0 + 1;
      int s0, mn0, s1, mn1;
      scale_min_k4(2 * k, sc, &s0, &mn0);
      scale_min_k4(2 * k + 1, sc, &s1, &mn1);
      acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(madd_u8i8(lo, ld(q + b0 * 32))),
                            _mm256_set1_ps(dd * (float)s0 * d[b0]), acc);
      acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(madd_u8i8(hi, ld(q + b1 * 32))),
                            _mm256_set1_ps(dd * (float)s1 * d[b1]), acc);
      mins = mins + dmin * ((float)mn0 * d[b0] * (float)(s16[2 * b0] + s16[2 * b0 + 1]) +
                            (float)mn1 * d[b1] * (float)(s16[2 * b1] + s16[2 * b1 + 1]));
    }
  }
  return hsum(acc) - mins;
}

// The four 6-bit runs of one 128-element half of a Q6_K superblock, as
// unsigned bytes (avx2.rs:128-133 / 399-404).
inline void q6_runs(const uint8_t* blk, int h, __m256i r[4]) {
  const __m256i m4 = _mm256_set1_epi8(0x0F), m3 = _mm256_set1_epi8(0x03);
  __m256i qh = ld(blk + 128 + h * 32);
  __m256i qa = ld(blk + h * 64), qb = ld(blk + h * 64 + 32);
  r[0] = _mm256_or_si256(_mm256_and_si256(qa, m4), _mm256_slli_epi16(_mm256_and_si256(qh, m3), 4));
  r[1] = _mm256_or_si256(_mm256_and_si256(qb, m4),
                         _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, 2), m3), 4));
  r[2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(qa, 4), m4),
                         _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, 4), m3), 4));
  r[3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(qb, 4), m4),
                         _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, 6), m3), 4));
}

float dot_q6_k_q8(const uint8_t* w, int64_t n, const int8_t* q, const float* d, const int32_t* s16) {
  __m256 acc = _mm256_setzero_ps();
  float offs = 0.f;
  for (int64_t sb = 0; sb < n / 256; ++sb) {
    const uint8_t* blk = w + sb * 210;
    float dd = h2f(blk + 208);
    for (int h = 0; h < 2; ++h) {
      __m256i r[4];
      q6_runs(blk, h, r);
      const int8_t* s = (const int8_t*)(blk + 192 + h * 8);
      for (int ri = 0; ri < 4; ++ri) {
        int64_t b = sb * 8 + h * 4 + ri;
        float lo = dd * (float)s[2 * ri] * d[b];
        float hi = dd * (float)s[2 * ri + 1] * d[b];
        __m256 sc = _mm256_set_m128(_mm_set1_ps(hi), _mm_set1_ps(lo));
        acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(madd_u8i8(r[ri], ld(q + b * 32))), sc, acc);
        offs = offs + 32.0f * (lo * (float)s16[2 * b] + hi * (float)s16[2 * b + 1]);
      }
    }
  }
  return hsum(acc) - offs;
}

// qdot::unpack (qdot.rs:75-184): int8 values with per-16 scale and min.
void unpack(int t, const uint8_t* w, int64_t n, int8_t* q, float* sc, float* mn) {
  switch (t) {
    case T_Q8_0:
      for (int64_t b = 0; b < n / 32; ++b) {
        const uint8_t* blk = w + b * 34;
        float d = h2f(blk);
        for (int j = 0; j < 32; ++j) q[b * 32 + j] = (int8_t)blk[2 + j];
        sc[2 * b] = d; sc[2 * b + 1] = d;
        mn[2 * b] = 0.f; mn[2 * b + 1] = 0.f;
      }
      return;
    case T_Q4_0:
    case T_Q4_1: {
      bool zero = t == T_Q4_0;
      int bs = zero ? 18 : 20, off = zero ? 2 : 4;
      for (int64_t b = 0; b < n / 32; ++b) {
        const uint8_t* blk = w + b * bs;
        float d = h2f(blk);
        int bias = zero ? 8 : 0;
        float m = zero ? 0.f : -h2f(blk + 2);
        for (int j = 0; j < 16; ++j) {
          q[b * 32 + j] = (int8_t)((blk[off + j] & 0xF) - bias);
          q[b * 32 + j + 16] = (int8_t)((blk[off + j] >> 4) - bias);
        }
        sc[2 * b] = d; sc[2 * b + 1] = d;
        mn[2 * b] = m; mn[2 * b + 1] = m;
      }
      return;
    }
    case T_Q5_0:
    case T_Q5_1: {
      bool zero = t == T_Q5_0;
      int bs = zero ? 22 : 24, off = zero ? 2 : 4;
      for (int64_t b = 0; b < n / 32; ++b) {
        const uint8_t* blk = w + b * bs;
        float d = h2f(blk);
        int bias = zero ? 16 : 0;
        float m = zero ? 0.f : -h2f(blk + 2);
        uint32_t qh;
        std::memcpy(&qh, blk + off, 4);
        const uint8_t* qs = blk + off + 4;
        for (int j = 0; j < 16; ++j) {
          uint8_t h0 = (uint8_t)(((qh >> j) << 4) & 0x10);
          uint8_t h1 = (uint8_t)((qh >> (j + 12)) & 0x10);
          q[b * 32 + j] = (int8_t)(((qs[j] & 0xF) | h0) - bias);
          q[b * 32 + j + 16] = (int8_t)(((qs[j] >> 4) | h1) - bias);
        }
        sc[2 * b] = d; sc[2 * b + 1] = d;
        mn[2 * b] = m; mn[2 * b + 1] = m;
      }
      return;
    }
    case T_Q4_K:
    case T_Q5_K: {
      bool k5 = t == T_Q5_K;
      int bs = k5 ? 176 : 144;
      for (int64_t sb = 0; sb < n / 256; ++sb) {
        const uint8_t* blk = w + sb * bs;
        float d = h2f(blk), dmin = h2f(blk + 2);
        const uint8_t* scales = blk + 4;
        const uint8_t* qh = blk + 16;
        const uint8_t* qs = k5 ? blk + 48 : blk + 16;
        for (int k = 0; k < 4; ++k) {
          int64_t base = sb * 256 + k * 64;
          for (int j = 0; j < 32; ++j) {
            uint8_t lo = qs[k * 32 + j] & 0xF, hi = qs[k * 32 + j] >> 4;
            if (k5) {
              lo |= ((qh[j] >> (2 * k)) & 1) << 4;
              hi |= ((qh[j] >> (2 * k + 1)) & 1) << 4;
            }
            q[base + j] = (int8_t)lo;
            q[base + 32 + j] = (int8_t)hi;
          }
          int s0, m0, s1, m1;
          scale_min_k4(2 * k, scales, &s0, &m0);
          scale_min_k4(2 * k + 1, scales, &s1, &m1);
          int64_t i16 = base / 16;
          for (int h = 0; h < 2; ++h) {
            sc[i16 + h] = d * (float)s0;
            mn[i16 + h] = dmin * (float)m0;
            sc[i16 + 2 + h] = d * (float)s1;
            mn[i16 + 2 + h] = dmin * (float)m1;
          }
        }
      }
      return;
    }
    case T_Q6_K:
      for (int64_t sb = 0; sb < n / 256; ++sb) {
        const uint8_t* blk = w + sb * 210;
        float d = h2f(blk + 208);
        for (int h = 0; h < 2; ++h) {
          const uint8_t* ql = blk + h * 64;
          const uint8_t* qh = blk + 128 + h * 32;
          const int8_t* s = (const int8_t*)(blk + 192 + h * 8);
          int64_t base = sb * 256 + h * 128;
          for (int l = 0; l < 32; ++l) {
            q[base + l] = (int8_t)(((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32);
            q[base + l + 32] = (int8_t)(((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32);
            q[base + l + 64] = (int8_t)(((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
            q[base + l + 96] = (int8_t)(((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
          }
          for (int r = 0; r < 4; ++r)
            for (int hf = 0; hf < 2; ++hf) {
              int64_t i16 = (base + 32 * r + 16 * hf) / 16;
              sc[i16] = d * (float)s[2 * r + hf];
              mn[i16] = 0.f;
            }
        }
      }
      return;
    default:
      return;
  }
}

// avx2::dot_unpacked (avx2.rs:150-164).
float dot_unpacked(const int8_t* uq, const float* usc, const float* umn, int64_t n, const int8_t* q,
                   const float* d, const int32_t* s16) {
  __m256 acc = _mm256_setzero_ps();
  float mins = 0.f;
  for (int64_t b = 0; b < n / 32; ++b) {
    __m256 p = _mm256_cvtepi32_ps(madd_i8i8(ld(uq + b * 32), ld(q + b * 32)));
    __m256 sc = _mm256_set_m128(_mm_set1_ps(usc[2 * b + 1] * d[b]), _mm_set1_ps(usc[2 * b] * d[b]));
    acc = _mm256_fmadd_ps(p, sc, acc);
    mins = mins + d[b] * (umn[2 * b] * (float)s16[2 * b] + umn[2 * b + 1] * (float)s16[2 * b + 1]);
  }
  return hsum(acc) - mins;
}

// qdot::dot_impl (qdot.rs:187-200): the portable scalar reference.
float dot_unpacked_scalar(const int8_t* uq, const float* usc, const float* umn, int64_t n, const int8_t* q,
                          const float* d, const int32_t* s16) {
  float sum = 0.f;
  for (int64_t k = 0; k < n / 16; ++k) {
    int32_t p = 0;
    for (int j = 0; j < 16; ++j) p += (int32_t)uq[k * 16 + j] * (int32_t)q[k * 16 + j];
    sum = sum + d[k / 2] * (usc[k] * (float)p - umn[k] * (float)s16[k]);
  }
  return sum;
}

// ---------------------------------------------------------------------------
// Q8_K kernels (avx2.rs:348-419).
float dot_q4_k_8k(const uint8_t* w, int64_t n, const int8_t* q, const float* xd, const int32_t* bsums) {
  const __m256i m4 = _mm256_set1_epi8(0x0F);
  __m256 acc = _mm256_setzero_ps();
  float summs = 0.f;
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* blk = w + b * 144;
    float d = h2f(blk) * xd[b];
    float dmin = h2f(blk + 2) * xd[b];
    const uint8_t* sc = blk + 4;
    const int8_t* xq = q + b * 256;
    __m256i sumi = _mm256_setzero_si256();
    int32_t mins = 0;
    for (int k = 0; k < 4; ++k) {
      int s0, m0, s1, m1;
      scale_min_k4(2 * k, sc, &s0, &m0);
      scale_min_k4(2 * k + 1, sc, &s1, &m1);
      __m256i v = ld(blk + 16 + 32 * k);
      __m256i lo = _mm256_and_si256(v, m4);
      __m256i hi = _mm256_and_si256(_mm256_srli_epi16(v, 4), m4);
      __m256i p0 = _mm256_madd_epi16(_mm256_maddubs_epi16(lo, ld(xq + 64 * k)), _mm256_set1_epi16((short)s0));
      __m256i p1 = _mm256_madd_epi16(_mm256_maddubs_epi16(hi, ld(xq + 64 * k + 32)), _mm256_set1_epi16((short)s1));
      sumi = _mm256_add_epi32(sumi, _mm256_add_epi32(p0, p1));
      const int32_t* bs = bsums + b * 16 + 4 * k;
      mins += m0 * (bs[0] + bs[1]) + m1 * (bs[2] + bs[3]);
    }
    acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(sumi), _mm256_set1_ps(d), acc);
    summs = summs + dmin * (float)mins;
  }
  return hsum(acc) - summs;
}

float dot_q6_k_8k(const uint8_t* w, int64_t n, const int8_t* q, const float* xd, const int32_t* bsums) {
  __m256 acc = _mm256_setzero_ps();
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* blk = w + b * 210;
    float d = h2f(blk + 208) * xd[b];
    const int8_t* xq = q + b * 256;
    __m256i sumi = _mm256_setzero_si256();
    int32_t offs = 0;
    for (int h = 0; h < 2; ++h) {
      __m256i r[4];
      q6_runs(blk, h, r);
      const int8_t* sc = (const int8_t*)(blk + 192 + h * 8);
      for (int ri = 0; ri < 4; ++ri) {
        short s0 = sc[2 * ri], s1 = sc[2 * ri + 1];
        __m256i p = _mm256_madd_epi16(_mm256_maddubs_epi16(r[ri], ld(xq + h * 128 + ri * 32)),
                                      _mm256_set_m128i(_mm_set1_epi16(s1), _mm_set1_epi16(s0)));
        sumi = _mm256_add_epi32(sumi, p);
        int64_t k16 = b * 16 + h * 8 + ri * 2;
        offs += (int32_t)s0 * bsums[k16] + (int32_t)s1 * bsums[k16 + 1];
      }
    }
    acc = _mm256_fmadd_ps(_mm256_cvtepi32_ps(sumi), _mm256_set1_ps(d), acc);
    acc = _mm256_add_ps(acc, _mm256_set_ps(0, 0, 0, 0, 0, 0, 0, -32.0f * d * (float)offs));
  }
  return hsum(acc);
}

// ---------------------------------------------------------------------------
// Lane emulations: the eight 32-bit lanes of the AVX2 kernels computed with
// plain integer loops. Lane j of a 32-byte run covers bytes 4j..4j+3; in the
// Q6_K kernel lanes 0-3 take the run's first sub-block scale, lanes 4-7 the
// second. These are the exact integer quantities the CUDA kernels reproduce.

// Q4_K x Q8_K, superblock `b`: sumi[8] and the integer min term.
void lanes_q4_k(const uint8_t* blk, const int8_t* xq, const int32_t* bs16, int32_t sumi[8], int32_t* mins) {
  const uint8_t* sc = blk + 4;
  const uint8_t* qs = blk + 16;
  for (int j = 0; j < 8; ++j) sumi[j] = 0;
  *mins = 0;
  for (int k = 0; k < 4; ++k) {
    int s0, m0, s1, m1;
    scale_min_k4(2 * k, sc, &s0, &m0);
    scale_min_k4(2 * k + 1, sc, &s1, &m1);
    for (int j = 0; j < 8; ++j) {
      int32_t plo = 0, phi = 0;
      for (int i = 4 * j; i < 4 * j + 4; ++i) {
        plo += (int32_t)(qs[32 * k + i] & 0xF) * xq[64 * k + i];
        phi += (int32_t)(qs[32 * k + i] >> 4) * xq[64 * k + 32 + i];
      }
      sumi[j] += s0 * plo + s1 * phi;
    }
    *mins += m0 * (bs16[4 * k] + bs16[4 * k + 1]) + m1 * (bs16[4 * k + 2] + bs16[4 * k + 3]);
  }
}

inline int q6_val(const uint8_t* blk, int h, int ri, int i) {
  const uint8_t* ql = blk + h * 64;
  const uint8_t* qh = blk + 128 + h * 32;
  int lowsrc = (ri & 1) ? ql[32 + i] : ql[i];
  int nib = (ri < 2) ? (lowsrc & 0xF) : (lowsrc >> 4);
  return nib | (((qh[i] >> (2 * ri)) & 3) << 4);
}

// Q6_K x Q8_K, superblock `b`: sumi[8] and the integer offset term.
void lanes_q6_k(const uint8_t* blk, const int8_t* xq, const int32_t* bs16, int32_t sumi[8], int32_t* offs) {
  for (int j = 0; j < 8; ++j) sumi[j] = 0;
  *offs = 0;
  for (int h = 0; h < 2; ++h) {
    const int8_t* sc = (const int8_t*)(blk + 192 + h * 8);
    for (int ri = 0; ri < 4; ++ri) {
      int s0 = sc[2 * ri], s1 = sc[2 * ri + 1];
      for (int j = 0; j < 8; ++j) {
        int32_t p = 0;
        for (int i = 4 * j; i < 4 * j + 4; ++i) p += q6_val(blk, h, ri, i) * xq[h * 128 + ri * 32 + i];
        sumi[j] += (j < 4 ? s0 : s1) * p;
      }
      int k16 = h * 8 + ri * 2;
      *offs += s0 * bs16[k16] + s1 * bs16[k16 + 1];
    }
  }
}

float dot_q4_k_8k_lanes(const uint8_t* w, int64_t n, const int8_t* q, const float* xd, const int32_t* bsums) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float summs = 0.f;
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* blk = w + b * 144;
    float d = h2f(blk) * xd[b];
    float dmin = h2f(blk + 2) * xd[b];
    int32_t sumi[8], mins;
    lanes_q4_k(blk, q + b * 256, bsums + b * 16, sumi, &mins);
    for (int j = 0; j < 8; ++j) acc[j] = std::fma((float)sumi[j], d, acc[j]);
    summs = summs + dmin * (float)mins;
  }
  return hsum8(acc) - summs;
}

float dot_q6_k_8k_lanes(const uint8_t* w, int64_t n, const int8_t* q, const float* xd, const int32_t* bsums) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int64_t b = 0; b < n / 256; ++b) {
    const uint8_t* blk = w + b * 210;
    float d = h2f(blk + 208) * xd[b];
    int32_t sumi[8], offs;
    lanes_q6_k(blk, q + b * 256, bsums + b * 16, sumi, &offs);
    for (int j = 0; j < 8; ++j) acc[j] = std::fma((float)sumi[j], d, acc[j]);
    // avx2.rs:416 adds a vector whose lanes 1..7 are +0.0 (turns -0.0 into +0.0).
    acc[0] = acc[0] + -32.0f * d * (float)offs;
    for (int j = 1; j < 8; ++j) acc[j] = acc[j] + 0.0f;
  }
  return hsum8(acc);
}

// Q8_0 x Q8Row lanes: lane j = sum of w*x over bytes 4j..4j+3 (the sign trick
// of avx2.rs:37-41 computes exactly w*x).
float dot_q8_0_lanes(const uint8_t* w, int64_t n, const int8_t* q, const float* d) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int64_t b = 0; b < n / 32; ++b) {
    const uint8_t* blk = w + b * 34;
    float s = h2f(blk) * d[b];
    for (int j = 0; j < 8; ++j) {
      int32_t p = 0;
      for (int i = 4 * j; i < 4 * j + 4; ++i) p += (int32_t)(int8_t)blk[2 + i] * q[b * 32 + i];
      acc[j] = std::fma((float)p, s, acc[j]);
    }
  }
  return hsum8(acc);
}

// ---------------------------------------------------------------------------
// gemm_f32 / dot_f32 (avx2.rs:226-308).
float dot_f32(const float* a, const float* b, int64_t n) {
  __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
  int64_t c = 0;
  for (; c + 16 <= n; c += 16) {
    acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + c), _mm256_loadu_ps(b + c), acc0);
    acc1 = _mm256_fmadd_ps(_mm256_loadu_ps(a + c + 8), _mm256_loadu_ps(b + c + 8), acc1);
  }
  for (; c + 8 <= n; c += 8) acc0 = _mm256_fmadd_ps(_mm256_loadu_ps(a + c), _mm256_loadu_ps(b + c), acc0);
  float s = hsum(_mm256_add_ps(acc0, acc1));
  for (; c < n; ++c) s = s + a[c] * b[c];
  return s;
}

void gemm_f32(const float* w, int64_t rows, const float* x, int64_t s_rows, int64_t cols, float* res) {
  int64_t rows3 = rows / 3 * 3;
  int64_t s = 0;
  for (; s + 4 <= s_rows; s += 4) {
    const float* xs[4] = {x + s * cols, x + (s + 1) * cols, x + (s + 2) * cols, x + (s + 3) * cols};
    for (int64_t r = 0; r < rows3; r += 3) {
      __m256 acc[12];
      for (auto& a : acc) a = _mm256_setzero_ps();
      const float* w0 = w + r * cols;
      const float* w1 = w0 + cols;
      const float* w2 = w1 + cols;
      for (int64_t c = 0; c < cols; c += 8) {
        __m256 a0 = _mm256_loadu_ps(w0 + c), a1 = _mm256_loadu_ps(w1 + c), a2 = _mm256_loadu_ps(w2 + c);
        for (int si = 0; si < 4; ++si) {
          __m256 b = _mm256_loadu_ps(xs[si] + c);
          acc[si * 3 + 0] = _mm256_fmadd_ps(a0, b, acc[si * 3 + 0]);
          acc[si * 3 + 1] = _mm256_fmadd_ps(a1, b, acc[si * 3 + 1]);
          acc[si * 3 + 2] = _mm256_fmadd_ps(a2, b, acc[si * 3 + 2]);
        }
      }
      for (int si = 0; si < 4; ++si)
        for (int ri = 0; ri < 3; ++ri) res[(r + ri) * s_rows + s + si] = hsum(acc[si * 3 + ri]);
    }
    for (int64_t r = rows3; r < rows; ++r)
      for (int si = 0; si < 4; ++si) res[r * s_rows + s + si] = dot_f32(w + r * cols, xs[si], cols);
  }
  for (; s < s_rows; ++s)
    for (int64_t r = 0; r < rows; ++r) res[r * s_rows + s] = dot_f32(w + r * cols, x + s * cols, cols);
}

// Scalar statement of one gemm_f32 output: the 8-lane FMA chain over c in
// steps of 8 followed by hsum (avx2.rs:245-270).
float lane_chain_f32(const float* a, const float* b, int64_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int64_t c = 0; c < n; c += 8)
    for (int j = 0; j < 8; ++j) acc[j] = std::fma(a[c + j], b[c + j], acc[j]);
  return hsum8(acc);
}

// ---------------------------------------------------------------------------
// quant::matmul (quant.rs:229-339): out[s][r] = W[r] . x[s].
bool g_exact = false;

bool qdot_supports(int t) {
  return t == T_Q8_0 || t == T_Q4_0 || t == T_Q4_1 || t == T_Q5_0 || t == T_Q5_1 || t == T_Q4_K ||
         t == T_Q5_K || t == T_Q6_K;
}

int matmul(int t, const uint8_t* w, int64_t rows, int64_t cols, const float* x, int64_t s_rows, float* out,
           bool exact) {
  int64_t row_bytes = bytes_for(t, cols);
  if (row_bytes < 0) return -1;
  const int64_t TILE = 16;
  auto scatter = [&](int64_t r0, int64_t r1, const std::vector<float>& res) {
    for (int64_t i = 0; i < r1 - r0; ++i)
      for (int64_t s = 0; s < s_rows; ++s) out[s * rows + r0 + i] = res[i * s_rows + s];
  };
  if (s_rows >= 4 && cols % 8 == 0) {
    const int64_t GT = 48;
    parallel_for((rows + GT - 1) / GT, [&](int64_t ti) {
      int64_t r0 = ti * GT, r1 = std::min(r0 + GT, rows);
      std::vector<float> wf((r1 - r0) * cols);
      for (int64_t r = r0; r < r1; ++r) dequant_row(t, w + r * row_bytes, cols, wf.data() + (r - r0) * cols);
      std::vector<float> res((r1 - r0) * s_rows);
      gemm_f32(wf.data(), r1 - r0, x, s_rows, cols, res.data());
      scatter(r0, r1, res);
    });
    return 0;
  }
  if (!exact && (t == T_Q4_K || t == T_Q6_K) && cols % 256 == 0) {
    std::vector<int8_t> q(s_rows * cols);
    std::vector<float> d(s_rows * cols / 256);
    std::vector<int32_t> bs(s_rows * cols / 16);
    for (int64_t s = 0; s < s_rows; ++s)
      q8k_quantize(x + s * cols, cols, q.data() + s * cols, d.data() + s * cols / 256, bs.data() + s * cols / 16);
    parallel_for((rows + TILE - 1) / TILE, [&](int64_t ti) {
      int64_t r0 = ti * TILE, r1 = std::min(r0 + TILE, rows);
      std::vector<float> res((r1 - r0) * s_rows);
      for (int64_t r = r0; r < r1; ++r)
        for (int64_t s = 0; s < s_rows; ++s) {
          const uint8_t* wr = w + r * row_bytes;
          const int8_t* qs = q.data() + s * cols;
          const float* ds = d.data() + s * cols / 256;
          const int32_t* bss = bs.data() + s * cols / 16;
          res[(r - r0) * s_rows + s] = t == T_Q4_K ? dot_q4_k_8k(wr, cols, qs, ds, bss)
                                                   : dot_q6_k_8k(wr, cols, qs, ds, bss);
        }
      scatter(r0, r1, res);
    });
    return 0;
  }
  if (!exact && qdot_supports(t) && cols % 32 == 0) {
    std::vector<int8_t> q(s_rows * cols);
    std::vector<float> d(s_rows * cols / 32);
    std::vector<int32_t> s16(s_rows * cols / 16);
    for (int64_t s = 0; s < s_rows; ++s)
      q8_quantize(x + s * cols, cols, q.data() + s * cols, d.data() + s * cols / 32, s16.data() + s * cols / 16);
    bool fused = t == T_Q8_0 || t == T_Q4_0 || t == T_Q4_K || t == T_Q6_K;
    parallel_for((rows + TILE - 1) / TILE, [&](int64_t ti) {
      int64_t r0 = ti * TILE, r1 = std::min(r0 + TILE, rows);
      std::vector<float> res((r1 - r0) * s_rows);
      std::vector<int8_t> uq(cols);
      std::vector<float> usc(cols / 16), umn(cols / 16);
      for (int64_t r = r0; r < r1; ++r) {
        const uint8_t* wr = w + r * row_bytes;
        if (!fused) unpack(t, wr, cols, uq.data(), usc.data(), umn.data());
        for (int64_t s = 0; s < s_rows; ++s) {
          const int8_t* qs = q.data() + s * cols;
          const float* ds = d.data() + s * cols / 32;
          const int32_t* ss = s16.data() + s * cols / 16;
          float v;
          if (!fused) v = dot_unpacked(uq.data(), usc.data(), umn.data(), cols, qs, ds, ss);
          else if (t == T_Q8_0) v = dot_q8_0(wr, cols, qs, ds);
          else if (t == T_Q4_0) v = dot_q4_0(wr, cols, qs, ds);
          else if (t == T_Q4_K) v = dot_q4_k_q8(wr, cols, qs, ds, ss);
          else v = dot_q6_k_q8(wr, cols, qs, ds, ss);
          res[(r - r0) * s_rows + s] = v;
        }
      }
      scatter(r0, r1, res);
    });
    return 0;
  }
  parallel_for((rows + TILE - 1) / TILE, [&](int64_t ti) {
    int64_t r0 = ti * TILE, r1 = std::min(r0 + TILE, rows);
    std::vector<float> buf(cols), res((r1 - r0) * s_rows);
    for (int64_t r = r0; r < r1; ++r) {
      dequant_row(t, w + r * row_bytes, cols, buf.data());
      for (int64_t s = 0; s < s_rows; ++s) res[(r - r0) * s_rows + s] = dot_scalar(buf.data(), x + s * cols, cols);
    }
    scatter(r0, r1, res);
  });
  return 0;
}

// ---------------------------------------------------------------------------
// Transformer::route (transformer.rs:472-496) on precomputed logits.
void route_rows(const float* logits, int64_t n_tok, int E, int k, bool norm_topk, float weights_scale,
                int32_t* ids, float* wts) {
  std::vector<float> p(E);
  std::vector<int> idx(E);
  for (int64_t s = 0; s < n_tok; ++s) {
    const float* row = logits + s * E;
    float m = -INFINITY;
    for (int e = 0; e < E; ++e) m = std::fmax(m, row[e]);
    for (int e = 0; e < E; ++e) p[e] = std::exp(row[e] - m);
    float sum = -0.0f;
    for (int e = 0; e < E; ++e) sum = sum + p[e];
    for (int e = 0; e < E; ++e) p[e] = p[e] / sum;
    for (int e = 0; e < E; ++e) idx[e] = e;
    std::stable_sort(idx.begin(), idx.end(), [&](int a, int b) {
      if (p[b] < p[a]) return true;   // descending by p
      if (p[a] < p[b]) return false;
      return a < b;                   // ties (and NaN) by index
    });
    float sel[64];
    for (int j = 0; j < k; ++j) sel[j] = p[idx[j]];
    if (norm_topk) {
      float ss = -0.0f;
      for (int j = 0; j < k; ++j) ss = ss + sel[j];
      ss = std::fmax(ss, 6.1035156e-5f);
      for (int j = 0; j < k; ++j) sel[j] = sel[j] / ss;
    }
    if (weights_scale != 0.f && weights_scale != 1.f)
      for (int j = 0; j < k; ++j) sel[j] = sel[j] * weights_scale;
    for (int j = 0; j < k; ++j) {
      ids[s * k + j] = idx[j];
      wts[s * k + j] = sel[j];
    }
  }
}

inline float silu_mul(float g, float u) { return g / (1.0f + std::exp(-g)) * u; }

}  // namespace

extern "C" int ko_moe_ffn(const float* h, int64_t n_tok, int64_t d, const float* router_w, int E, int k, int norm_topk,
               float weights_scale, int t_gate, const uint8_t* gate, int t_up, const uint8_t* up, int t_down,
               const uint8_t* down, int64_t ff, float* out, int32_t* ids_out, float* w_out, int t_sh_gate,
               const uint8_t* sh_gate, int t_sh_up, const uint8_t* sh_up, int t_sh_down, const uint8_t* sh_down,
               int64_t sh_ff, const float* sh_inp);

namespace {
// ---------------------------------------------------------------------------
// Transformer::forward (transformer.rs:287-302, 360-467) for llama / qwen2 /
// qwen3 and their MoE variants, every weight resident in host memory (the
// pointers given to ko_model_set are kept, not copied). Tensor kinds of a
// layer (KO_*) and of the model (KO_G_*) share their numbering with the CUDA
// library's kc_model_tensor.
enum {
  KO_ATTN_NORM = 0, KO_WQ, KO_WK, KO_WV, KO_WO, KO_BQ, KO_BK, KO_BV, KO_QNORM, KO_KNORM, KO_FFN_NORM,
  KO_GATE, KO_UP, KO_DOWN, KO_ROUTER, KO_GATE_EXPS, KO_UP_EXPS, KO_DOWN_EXPS, KO_SH_GATE, KO_SH_UP,
  KO_SH_DOWN, KO_SH_INP, KO_N_LAYER_T
};
enum { KO_G_EMBD = 0, KO_G_OUT_NORM = 1, KO_G_OUTPUT = 2, KO_N_G = 3 };

struct OTensor {
  int t = -1;
  const uint8_t* w = nullptr;
  int64_t rows = 0, cols = 0;
};

struct OModel {
  int n_layer = 0, d = 0, n_head = 0, n_kv = 0, hd = 0, n_vocab = 0, n_ctx = 0, rope_dim = 0;
  float eps = 0.f;
  bool neox = true;
  int n_expert = 0, k = 0;
  bool norm_topk = true;
  float weights_scale = 0.f;
  std::vector<float> inv_freq;
  std::vector<std::vector<OTensor>> layers;
  OTensor g[KO_N_G];
  std::vector<std::vector<uint16_t>> kc, vc;  // f16 bits [n_ctx][n_kv * hd] per layer
  int cached = 0;
};

// Transformer::vec_of: a small tensor dequantised to f32.
std::vector<float> vec_of(const OTensor& t) {
  std::vector<float> v(t.rows * t.cols);
  const int64_t rb = bytes_for(t.t, t.cols);
  for (int64_t r = 0; r < t.rows; ++r) dequant_row(t.t, t.w + r * rb, t.cols, v.data() + r * t.cols);
  return v;
}

std::vector<float> mm(const OTensor& t, const std::vector<float>& x) {
  const int64_t s = (int64_t)x.size() / t.cols;
  std::vector<float> out(s * t.rows);
  matmul(t.t, t.w, t.rows, t.cols, x.data(), s, out.data(), g_exact);
  return out;
}

// Transformer::rmsnorm (transformer.rs:330-340): sum of squares folded in
// order from -0.0, divided by dim, r = 1 / sqrt(ss + eps), then x * r * w.
std::vector<float> rmsnorm(const float* x, int64_t n, const std::vector<float>& w, int64_t dim, float eps) {
  std::vector<float> out(n);
  for (int64_t r0 = 0; r0 < n; r0 += dim) {
    float ss = -0.0f;
    for (int64_t j = 0; j < dim; ++j) ss = ss + x[r0 + j] * x[r0 + j];
    ss = ss / (float)dim;
    const float r = 1.0f / std::sqrt(ss + eps);
    for (int64_t j = 0; j < dim; ++j) out[r0 + j] = x[r0 + j] * r * w[j];
  }
  return out;
}

// Transformer::rope (transformer.rs:342-358).
void rope(const OModel& m, float* x, int64_t n, int n_heads, int pos0) {
  const int hd = m.hd, rd = m.rope_dim;
  const int64_t s_rows = n / ((int64_t)n_heads * hd);
  for (int64_t s = 0; s < s_rows; ++s) {
    const float p = (float)(pos0 + s);
    for (int h = 0; h < n_heads; ++h) {
      float* v = x + (s * n_heads + h) * hd;
      for (int i = 0; i < rd / 2; ++i) {
        const float a_ = p * m.inv_freq[i];
        const float sn = std::sin(a_), cs = std::cos(a_);
        const int a = m.neox ? i : 2 * i, b = m.neox ? i + rd / 2 : 2 * i + 1;
        const float x0 = v[a], x1 = v[b];
        v[a] = x0 * cs - x1 * sn;
        v[b] = x0 * sn + x1 * cs;
      }
    }
  }
}

uint16_t f2h(float f) { return _cvtss_sh(f, _MM_FROUND_TO_NEAREST_INT); }
float h2f16(uint16_t h) { return _cvtsh_ss(h); }

// Transformer::attention (transformer.rs:594-631): causal GQA over the f16
// cache; per (query, head) scores = dot * scale, max, exp, sum from +0.0,
// inv = 1 / sum, then o += (sc * inv) * v position by position.
std::vector<float> attention(const OModel& m, int l, const std::vector<float>& q, int pos0, int s_rows) {
  const int hd = m.hd, nh = m.n_head, nkv = m.n_kv, group = nh / nkv;
  const float scale = 1.0f / std::sqrt((float)hd);
  const int kvw = nkv * hd, n_tot = pos0 + s_rows;
  std::vector<float> kf((int64_t)n_tot * kvw), vf((int64_t)n_tot * kvw);
  for (int64_t i = 0; i < (int64_t)n_tot * kvw; ++i) {
    kf[i] = h2f16(m.kc[l][i]);
    vf[i] = h2f16(m.vc[l][i]);
  }
  std::vector<float> out((int64_t)s_rows * nh * hd, 0.f);
  parallel_for((int64_t)s_rows * nh, [&](int64_t i) {
    const int s = (int)(i / nh), h = (int)(i % nh), kvh = h / group;
    const float* qv = q.data() + ((int64_t)s * nh + h) * hd;
    const int n = pos0 + s + 1;
    std::vector<float> sc(n);
    for (int p = 0; p < n; ++p) sc[p] = dot_scalar(qv, kf.data() + (int64_t)p * kvw + kvh * hd, hd) * scale;
    float mx = -INFINITY;
    for (int p = 0; p < n; ++p) mx = std::fmax(mx, sc[p]);
    float sum = 0.0f;
    for (int p = 0; p < n; ++p) {
      sc[p] = std::exp(sc[p] - mx);
      sum = sum + sc[p];
    }
    const float inv = 1.0f / sum;
    float* o = out.data() + i * hd;
    for (int p = 0; p < n; ++p) {
      const float w = sc[p] * inv;
      const float* vr = vf.data() + (int64_t)p * kvw + kvh * hd;
      for (int j = 0; j < hd; ++j) o[j] = o[j] + w * vr[j];
    }
  });
  return out;
}

void add_into(std::vector<float>& x, const std::vector<float>& y) {
  for (size_t i = 0; i < x.size(); ++i) x[i] = x[i] + y[i];
}

// Transformer::forward_chunk_inner (transformer.rs:375-467) for one chunk.
int forward_chunk(OModel& m, const uint32_t* tokens, int s_rows, float* logits) {
  const int d = m.d, pos0 = m.cached;
  std::vector<float> x((int64_t)s_rows * d);
  const OTensor& E = m.g[KO_G_EMBD];
  const int64_t erb = bytes_for(E.t, d);
  for (int s = 0; s < s_rows; ++s) {
    if ((int)tokens[s] >= m.n_vocab) return -1;
    dequant_row(E.t, E.w + (int64_t)tokens[s] * erb, d, x.data() + (int64_t)s * d);  // quant::get_row
  }
  for (int l = 0; l < m.n_layer; ++l) {
    const auto& L = m.layers[l];
    {
      std::vector<float> h = rmsnorm(x.data(), (int64_t)x.size(), vec_of(L[KO_ATTN_NORM]), d, m.eps);
      std::vector<float> q = mm(L[KO_WQ], h), k = mm(L[KO_WK], h), v = mm(L[KO_WV], h);
      const int bias_kind[3] = {KO_BQ, KO_BK, KO_BV};
      std::vector<float>* ys[3] = {&q, &k, &v};
      for (int i = 0; i < 3; ++i)
        if (L[bias_kind[i]].w) {
          std::vector<float> b = vec_of(L[bias_kind[i]]);
          for (size_t r = 0; r < ys[i]->size(); ++r) (*ys[i])[r] = (*ys[i])[r] + b[r % b.size()];
        }
      if (L[KO_QNORM].w) q = rmsnorm(q.data(), (int64_t)q.size(), vec_of(L[KO_QNORM]), m.hd, m.eps);
      if (L[KO_KNORM].w) k = rmsnorm(k.data(), (int64_t)k.size(), vec_of(L[KO_KNORM]), m.hd, m.eps);
      rope(m, q.data(), (int64_t)q.size(), m.n_head, pos0);
      rope(m, k.data(), (int64_t)k.size(), m.n_kv, pos0);
      const int kvw = m.n_kv * m.hd;
      for (int s = 0; s < s_rows; ++s)
        for (int j = 0; j < kvw; ++j) {
          m.kc[l][(int64_t)(pos0 + s) * kvw + j] = f2h(k[(int64_t)s * kvw + j]);
          m.vc[l][(int64_t)(pos0 + s) * kvw + j] = f2h(v[(int64_t)s * kvw + j]);
        }
      std::vector<float> ctx = attention(m, l, q, pos0, s_rows);
      add_into(x, mm(L[KO_WO], ctx));
    }
    {
      std::vector<float> h = rmsnorm(x.data(), (int64_t)x.size(), vec_of(L[KO_FFN_NORM]), d, m.eps);
      std::vector<float> y((int64_t)s_rows * d);
      if (L[KO_ROUTER].w) {
        const OTensor &G = L[KO_GATE_EXPS], &U = L[KO_UP_EXPS], &D = L[KO_DOWN_EXPS];
        const int64_t ff = G.rows / m.n_expert;
        const OTensor &SG = L[KO_SH_GATE], &SU = L[KO_SH_UP], &SD = L[KO_SH_DOWN];
        std::vector<float> sh_inp;
        if (L[KO_SH_INP].w) sh_inp = vec_of(L[KO_SH_INP]);
        int rc = ko_moe_ffn(h.data(), s_rows, d, (const float*)L[KO_ROUTER].w, m.n_expert, m.k, m.norm_topk,
                            m.weights_scale, G.t, G.w, U.t, U.w, D.t, D.w, ff, y.data(), nullptr, nullptr, SG.t,
                            SG.w, SU.t, SU.w, SD.t, SD.w, SG.rows, sh_inp.empty() ? nullptr : sh_inp.data());
        if (rc) return rc;
      } else {
        std::vector<float> g = mm(L[KO_GATE], h), u = mm(L[KO_UP], h);
        for (size_t i = 0; i < g.size(); ++i) g[i] = silu_mul(g[i], u[i]);
        y = mm(L[KO_DOWN], g);
      }
      add_into(x, y);
    }
  }
  m.cached += s_rows;
  const float* last = x.data() + (int64_t)(s_rows - 1) * d;
  std::vector<float> normed = rmsnorm(last, d, vec_of(m.g[KO_G_OUT_NORM]), d, m.eps);
  const OTensor& O = m.g[KO_G_OUTPUT].w ? m.g[KO_G_OUTPUT] : m.g[KO_G_EMBD];  // tied embeddings
  std::vector<float> lg = mm(O, normed);
  std::memcpy(logits, lg.data(), lg.size() * 4);
  return 0;
}

}  // namespace

// ===========================================================================
// C ABI (ctypes). All pointers are host pointers; sizes in elements.
extern "C" {

void ko_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int ko_get_threads() { return g_threads; }
int ko_block_elems(int t) { return blk_elems(t); }
int ko_block_bytes(int t) { return blk_bytes(t); }
int64_t ko_bytes_for(int t, int64_t n) { return bytes_for(t, n); }
float ko_f16_to_f32(uint16_t h) {
  uint8_t b[2] = {(uint8_t)(h & 0xFF), (uint8_t)(h >> 8)};
  return h2f(b);
}

void ko_dequant_row(int t, const uint8_t* src, int64_t n, float* out) { dequant_row(t, src, n, out); }
float ko_dot(const float* a, const float* b, int64_t n) { return dot_scalar(a, b, n); }
float ko_dot_f32(const float* a, const float* b, int64_t n) { return dot_f32(a, b, n); }
float ko_lane_chain_f32(const float* a, const float* b, int64_t n) { return lane_chain_f32(a, b, n); }
void ko_gemm_f32(const float* w, int64_t rows, const float* x, int64_t s_rows, int64_t cols, float* res) {
  gemm_f32(w, rows, x, s_rows, cols, res);
}

void ko_q8_quantize(const float* x, int64_t n, int8_t* q, float* d, int32_t* s16) { q8_quantize(x, n, q, d, s16); }
void ko_q8k_quantize(const float* x, int64_t n, int8_t* q, float* d, int32_t* bsums) {
  q8k_quantize(x, n, q, d, bsums);
}

void ko_unpack(int t, const uint8_t* w, int64_t n, int8_t* q, float* sc, float* mn) { unpack(t, w, n, q, sc, mn); }
float ko_dot_unpacked(const int8_t* uq, const float* usc, const float* umn, int64_t n, const int8_t* q,
                      const float* d, const int32_t* s16) {
  return dot_unpacked(uq, usc, umn, n, q, d, s16);
}
float ko_dot_unpacked_scalar(const int8_t* uq, const float* usc, const float* umn, int64_t n, const int8_t* q,
                             const float* d, const int32_t* s16) {
  return dot_unpacked_scalar(uq, usc, umn, n, q, d, s16);
}

// Fused Q8Row kernels: t in {Q8_0, Q4_0, Q4_K, Q6_K}.
float ko_dot_fused(int t, const uint8_t* w, int64_t n, const int8_t* q, const float* d, const int32_t* s16) {
  switch (t) {
    case T_Q8_0: return dot_q8_0(w, n, q, d);
    case T_Q4_0: return dot_q4_0(w, n, q, d);
    case T_Q4_K: return dot_q4_k_q8(w, n, q, d, s16);
    case T_Q6_K: return dot_q6_k_q8(w, n, q, d, s16);
    default: return NAN;
  }
}
float ko_dot_q8_0_lanes(const uint8_t* w, int64_t n, const int8_t* q, const float* d) {
  return dot_q8_0_lanes(w, n, q, d);
}

// Q8_K kernels: t in {Q4_K, Q6_K}. `lanes` selects the scalar emulation.
float ko_dot_fused_k(int t, const uint8_t* w, int64_t n, const int8_t* q, const float* d, const int32_t* bsums,
                     int lanes) {
  if (t == T_Q4_K) return lanes ? dot_q4_k_8k_lanes(w, n, q, d, bsums) : dot_q4_k_8k(w, n, q, d, bsums);
  if (t == T_Q6_K) return lanes ? dot_q6_k_8k_lanes(w, n, q, d, bsums) : dot_q6_k_8k(w, n, q, d, bsums);
  return NAN;
}

// Per-superblock integer sums of a K-quant row against a Q8_K row:
// out[b*9 + j] = lane j (0..7) of sumi, out[b*9 + 8] = mins (Q4_K) / offs (Q6_K).
void ko_block_sums_k(int t, const uint8_t* w, int64_t n, const int8_t* q, const int32_t* bsums, int32_t* out) {
  for (int64_t b = 0; b < n / 256; ++b) {
    if (t == T_Q4_K) lanes_q4_k(w + b * 144, q + b * 256, bsums + b * 16, out + b * 9, out + b * 9 + 8);
    else lanes_q6_k(w + b * 210, q + b * 256, bsums + b * 16, out + b * 9, out + b * 9 + 8);
  }
}

void ko_set_exact(int on) { g_exact = on != 0; }

int ko_matmul(int t, const uint8_t* w, int64_t rows, int64_t cols, const float* x, int64_t s_rows, float* out) {
  return matmul(t, w, rows, cols, x, s_rows, out, g_exact);
}

void ko_route(const float* logits, int64_t n_tok, int E, int k, int norm_topk, float weights_scale, int32_t* ids,
              float* wts) {
  route_rows(logits, n_tok, E, k, norm_topk != 0, weights_scale, ids, wts);
}

// Transformer::moe_ffn (transformer.rs:513-589) for one layer with all
// experts resident. Stacked expert tensors: expert e's gate/up rows start at
// e * ff * row_bytes(d), its down rows at e * d * row_bytes(ff)
// (TensorInfo::slice_offset, crates/kestrel-gguf/src/lib.rs:183-189).
// router_w: F32 [E, d] (ffn_gate_inp.weight). Optional shared expert (qwen2moe,
// transformer.rs:571-587): sh_* may be null. Returns 0, or -1 on bad shapes.
int ko_moe_ffn(const float* h, int64_t n_tok, int64_t d, const float* router_w, int E, int k, int norm_topk,
               float weights_scale, int t_gate, const uint8_t* gate, int t_up, const uint8_t* up, int t_down,
               const uint8_t* down, int64_t ff, float* out, int32_t* ids_out, float* w_out, int t_sh_gate,
               const uint8_t* sh_gate, int t_sh_up, const uint8_t* sh_up, int t_sh_down, const uint8_t* sh_down,
               int64_t sh_ff, const float* sh_inp) {
  if (k < 1 || k > 64 || k > E) return -1;
  int64_t rb_g = bytes_for(t_gate, d), rb_u = bytes_for(t_up, d), rb_d = bytes_for(t_down, ff);
  if (rb_g < 0 || rb_u < 0 || rb_d < 0) return -1;
  std::vector<float> logits(n_tok * E);
  int rc = matmul(T_F32, (const uint8_t*)router_w, E, d, h, n_tok, logits.data(), g_exact);
  if (rc) return rc;
  std::vector<int32_t> ids(n_tok * k);
  std::vector<float> wts(n_tok * k);
  route_rows(logits.data(), n_tok, E, k, norm_topk != 0, weights_scale, ids.data(), wts.data());
  if (ids_out) std::memcpy(ids_out, ids.data(), ids.size() * 4);
  if (w_out) std::memcpy(w_out, wts.data(), wts.size() * 4);
  // assign: BTreeMap<expert, Vec<(token, w)>> in token order (:525-530).
  std::map<int, std::vector<std::pair<int64_t, float>>> assign;
  for (int64_t s = 0; s < n_tok; ++s)
    for (int j = 0; j < k; ++j) assign[ids[s * k + j]].push_back({s, wts[s * k + j]});
  std::map<int, std::vector<float>> ys;
  for (auto& [e, rows] : assign) {
    int64_t n = (int64_t)rows.size();
    std::vector<float> xs(n * d), g(n * ff), u(n * ff), y(n * d);
    for (int64_t i = 0; i < n; ++i) std::memcpy(xs.data() + i * d, h + rows[i].first * d, d * 4);
    matmul(t_gate, gate + (int64_t)e * ff * rb_g, ff, d, xs.data(), n, g.data(), g_exact);
    matmul(t_up, up + (int64_t)e * ff * rb_u, ff, d, xs.data(), n, u.data(), g_exact);
    for (int64_t i = 0; i < n * ff; ++i) g[i] = silu_mul(g[i], u[i]);
    matmul(t_down, down + (int64_t)e * d * rb_d, d, ff, g.data(), n, y.data(), g_exact);
    ys[e] = std::move(y);
  }
  std::fill(out, out + n_tok * d, 0.f);
  for (auto& [e, y] : ys) {  // ascending expert id (:566-570)
    auto& rows = assign[e];
    for (size_t i = 0; i < rows.size(); ++i) {
      float* o = out + rows[i].first * d;
      const float* yy = y.data() + i * d;
      float w = rows[i].second;
      for (int64_t c = 0; c < d; ++c) o[c] = o[c] + w * yy[c];
    }
  }
  if (sh_gate && sh_up && sh_down) {
    int64_t sg = sh_ff;
    std::vector<float> g(n_tok * sg), u(n_tok * sg), y(n_tok * d);
    matmul(t_sh_gate, sh_gate, sg, d, h, n_tok, g.data(), g_exact);
    matmul(t_sh_up, sh_up, sg, d, h, n_tok, u.data(), g_exact);
    for (int64_t i = 0; i < n_tok * sg; ++i) g[i] = silu_mul(g[i], u[i]);
    matmul(t_sh_down, sh_down, d, sg, g.data(), n_tok, y.data(), g_exact);
    for (int64_t s = 0; s < n_tok; ++s) {
      float gt = 1.0f;
      if (sh_inp) gt = 1.0f / (1.0f + std::exp(-dot_scalar(sh_inp, h + s * d, d)));
      for (int64_t c = 0; c < d; ++c) out[s * d + c] = out[s * d + c] + gt * y[s * d + c];
    }
  }
  return 0;
}

// One expert of Transformer::moe_ffn (transformer.rs:551-563): gate and up
// products of its n rows xs [n, d], g / (1 + exp(-g)) * u, then the down
// product -> y [n, d]. Matrices are one expert's rows. Returns 0, or -1 on
// bad shapes.
int ko_expert_ffn(int t_gate, const uint8_t* gate, int t_up, const uint8_t* up, int t_down, const uint8_t* down,
                  int64_t d, int64_t ff, const float* xs, int64_t n, float* y) {
  if (bytes_for(t_gate, d) < 0 || bytes_for(t_up, d) < 0 || bytes_for(t_down, ff) < 0) return -1;
  std::vector<float> g(n * ff), u(n * ff);
  if (int rc = matmul(t_gate, gate, ff, d, xs, n, g.data(), g_exact)) return rc;
  if (int rc = matmul(t_up, up, ff, d, xs, n, u.data(), g_exact)) return rc;
  for (int64_t i = 0; i < n * ff; ++i) g[i] = silu_mul(g[i], u[i]);
  return matmul(t_down, down, d, ff, g.data(), n, y, g_exact);
}

// ---- model (Transformer) ----------------------------------------------------
// arch: 0 llama (interleaved RoPE), 1 qwen2, 2 qwen3 (NeoX RoPE; transformer.rs:241).
void* ko_model_new(int n_layer, int d, int n_head, int n_kv, int head_dim, int n_vocab, int n_ctx, int rope_dim,
                   float rope_base, float eps, int arch, int n_expert, int k, int norm_topk, float weights_scale) {
  OModel* m = new OModel();
  m->n_layer = n_layer; m->d = d; m->n_head = n_head; m->n_kv = n_kv; m->hd = head_dim; m->n_vocab = n_vocab;
  m->n_ctx = n_ctx; m->rope_dim = rope_dim; m->eps = eps; m->neox = arch != 0;
  m->n_expert = n_expert; m->k = k; m->norm_topk = norm_topk != 0; m->weights_scale = weights_scale;
  for (int i = 0; i < rope_dim / 2; ++i)  // transformer.rs:248
    m->inv_freq.push_back(std::pow(rope_base, -(2.0f * (float)i) / (float)rope_dim));
  m->layers.assign(n_layer, std::vector<OTensor>(KO_N_LAYER_T));
  m->kc.assign(n_layer, std::vector<uint16_t>((int64_t)n_ctx * n_kv * head_dim, 0));
  m->vc.assign(n_layer, std::vector<uint16_t>((int64_t)n_ctx * n_kv * head_dim, 0));
  return m;
}
void ko_model_free(void* p) { delete (OModel*)p; }
// layer < 0: a model tensor (KO_G_*).
int ko_model_set(void* p, int layer, int kind, int t, const void* w, int64_t rows, int64_t cols) {
  OModel* m = (OModel*)p;
  OTensor T;
  T.t = t; T.w = (const uint8_t*)w; T.rows = rows; T.cols = cols;
  if (layer < 0) {
    if (kind < 0 || kind >= KO_N_G) return -1;
    m->g[kind] = T;
  } else {
    if (layer >= m->n_layer || kind < 0 || kind >= KO_N_LAYER_T) return -1;
    m->layers[layer][kind] = T;
  }
  return 0;
}
// Transformer::forward: feed tokens after the cached ones (chunks of
// n_batch = 256, transformer.rs:287-302); logits [n_vocab] of the last token.
int ko_model_forward(void* p, const uint32_t* tokens, int n, float* logits) {
  OModel* m = (OModel*)p;
  if (n < 1 || m->cached + n > m->n_ctx) return -2;
  for (int c = 0; c < n; c += 256) {
    int rc = forward_chunk(*m, tokens + c, std::min(256, n - c), logits);
    if (rc) return rc;
  }
  return 0;
}
void ko_model_truncate(void* p, int keep) {
  OModel* m = (OModel*)p;
  m->cached = std::min(m->cached, std::max(0, keep));
}

// sampler::argmax (sampler.rs:104-112): first maximum wins.
int ko_argmax(const float* l, int64_t n) {
  int64_t best = 0;
  for (int64_t i = 1; i < n; ++i)
    if (l[i] > l[best]) best = i;
  return (int)best;
}

}  // extern "C"
