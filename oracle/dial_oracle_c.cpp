/*
 * dial_oracle_c.cpp -- C++/OpenMP restatement of DIAL's decoder-layer path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the CPU
 * legs of bench.py load this library (through oracle/dial_oracle_fast.py);
 * the product (dial-27b_b200) never does and has no CPU fallback.
 *
 * It is the same algorithm as oracle/dial_oracle.py, function by function and
 * with the same rounding points, written so that the full Qwen3-8B-shape model
 * (36 layers, hidden 4096, vocab 151936) runs on host cores in seconds per
 * token.  Each function names the reference file:line it follows (paths are
 * relative to the reference project root, lisa301/DIAL-27B):
 *
 *   W8A16 row quantization ......... dial-core/src/models/qwen3_vl/worker_w8a16.rs:330-341
 *   W8A16 linear ................... dial-core/src/models/qwen3_vl/worker_w8a16.rs:146-224
 *   e2m1 / e4m3 decoders ........... dial-core/src/models/qwen3_8/cuda_quant.rs:11-41
 *   NVFP4 / FP8 linears ............ dial-core/src/models/qwen3_8/cuda_quant.rs:43-206
 *   RoPE tables .................... dial-core/src/models/llama3/cache.rs:37-67
 *   KV cache (append / replace) .... dial-core/src/models/llama3/cache.rs:117-237
 *   q/k norm, RoPE, attention ...... dial-core/src/models/qwen3_vl/text.rs:1143-1153,1258-1358,1478-1596
 *   SwiGLU MLP ..................... dial-core/src/models/qwen3_vl/text.rs:816-820
 *   pre-norm residual block ........ dial-core/src/models/qwen3_vl/text.rs:1636-1688
 *   embedding, head, greedy argmax . dial-core/src/models/qwen3_vl/qwen3_vl.rs:138-143,2459-2498,3302
 *
 * Rounding points (the ones dial_oracle.py fixes for the candle-owned ops):
 * every op output is rounded to bf16; RMSNorm m = bf16(sqrt(sum x^2 / n + eps)),
 * y = bf16(bf16(x / m) * w); RoPE three roundings; SiLU bf16(v / bf16(1 +
 * bf16(exp(-v)))) then bf16(s * u); attention scores bf16(bf16(q.k) *
 * bf16(1/sqrt(d))), softmax in f32 with probabilities rounded to bf16
 * (round_probs = 1) or kept in f32 (0), output bf16(sum p v).
 *
 * Matmul accumulation: `accum = 64` sums in f64 (the products of bf16
 * activations with int8 / bf16 weights are exact in f64 and their sums stay
 * exact for activations of ordinary magnitude, so the result does not depend
 * on summation order and equals dial_oracle.py's); `accum = 32` sums in f32
 * (the reference kernels' "f32 accumulate", used when this library is timed
 * as the CPU baseline).
 */
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

namespace {

typedef float v8f __attribute__((vector_size(32)));
typedef double v4d __attribute__((vector_size(32)));

inline float bits_to_f(uint32_t b) {
  float f;
  std::memcpy(&f, &b, 4);
  return f;
}
inline uint32_t f_to_bits(float f) {
  uint32_t b;
  std::memcpy(&b, &f, 4);
  return b;
}

// Round an f32 value to the nearest bf16 (ties to even), returned as f32.
inline float bf16r(float x) {
  if (std::isnan(x)) return x;
  uint64_t b = f_to_bits(x);
  b = (b + (((b >> 16) & 1u) + 0x7fffu)) & 0xffff0000u;
  return bits_to_f(static_cast<uint32_t>(b));
}
inline uint16_t bf16_bits(float x) { return static_cast<uint16_t>(f_to_bits(bf16r(x)) >> 16); }
inline float bf16_val(uint16_t b) { return bits_to_f(static_cast<uint32_t>(b) << 16); }

// ------------------------------------------------------------ synthetic data
// SplitMix64 finalizer of (seed, stream, index): the generator the engine's
// device fill (synth_table_fill) and dial_oracle.synth_hash share.
inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
inline uint64_t synth_base(uint64_t seed, uint64_t stream) {
  return (seed * 0x9E3779B97F4A7C15ull) ^ (stream * 0xD1B54A32D192ED03ull);
}
void synth_normal(uint64_t seed, uint64_t stream, int64_t n, const float* table, float* out) {
  const uint64_t base = synth_base(seed, stream);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = table[mix64(static_cast<uint64_t>(i) + base) & 0xffffu];
}

// ------------------------------------------------------------- e4m3 / e2m1
const float kE2m1[16] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f,
                         0.f, -0.5f, -1.f, -1.5f, -2.f, -3.f, -4.f, -6.f};

// Software e4m3 decode (cuda_quant.rs:27-41): subnormals m * 2^-9, the NaN
// codes 0x7F / 0xFF decode to 0.
float e4m3_decode(uint8_t c) {
  const int sign = c >> 7, ex = (c >> 3) & 15, man = c & 7;
  float v;
  if (ex == 0)
    v = static_cast<float>(man) * 0.001953125f;
  else
    v = std::ldexp(1.0f + static_cast<float>(man) * 0.125f, ex - 7);
  if (ex == 15 && man == 7) v = 0.f;
  return sign ? -v : v;
}

struct E4m3Table {
  float v[256];
  E4m3Table() {
    for (int i = 0; i < 256; ++i) v[i] = e4m3_decode(static_cast<uint8_t>(i));
  }
};
const E4m3Table& e4m3_table() {
  static E4m3Table t;
  return t;
}

// Nearest e4m3 code, ties to the even code, saturating at 448 (the encoder
// of dial_oracle.f32_to_e4m3, which builds FP8 test weights).
uint8_t f32_to_e4m3(float v) {
  const float* pos = e4m3_table().v;  // codes 0..126 ascending
  const float mag = std::min(std::fabs(v), 448.0f);
  if (mag == 0.f) return 0;
  int idx = static_cast<int>(std::lower_bound(pos, pos + 127, mag) - pos);
  idx = std::min(std::max(idx, 1), 126);
  const float lo = pos[idx - 1], hi = pos[idx];
  const float dlo = mag - lo, dhi = hi - mag;
  const bool pick_hi = dlo > dhi || (dlo == dhi && (idx & 1) == 0);
  uint8_t code = static_cast<uint8_t>(pick_hi ? idx : idx - 1);
  if (v < 0 && code != 0) code |= 0x80;
  return code;
}

// Nearest e2m1 code, ties to the smaller magnitude (dial_oracle.f32_to_e2m1).
uint8_t f32_to_e2m1(float v) {
  const float mag = std::min(std::fabs(v), 6.0f);
  int best = 0;
  float bd = std::fabs(mag - kE2m1[0]);
  for (int i = 1; i < 8; ++i) {
    const float d = std::fabs(mag - kE2m1[i]);
    if (d < bd) {
      bd = d;
      best = i;
    }
  }
  if (v < 0 && best != 0) best |= 0x8;
  return static_cast<uint8_t>(best);
}

// ------------------------------------------------------------------ linears
enum Fmt { kW8A16 = 0, kFp8Block128 = 1, kNvfp4 = 3, kDense = 4 };

struct Linear {
  int fmt = kW8A16;
  int64_t N = 0, K = 0;
  std::vector<int8_t> q;        // W8A16 codes [N][K]
  std::vector<float> s;         // W8A16 row scales [N]
  std::vector<uint8_t> codes;   // FP8 codes [N][K] or NVFP4 packed [N][K/2]
  std::vector<float> bscale;    // FP8 block scales [ceil(N/128)][ceil(K/128)]
  std::vector<uint8_t> gscale;  // NVFP4 e4m3 group scale codes [N][K/16]
  float global = 1.f;
  std::vector<uint16_t> dense;  // bf16 bits [N][K]

  // f32 value of weight row n (what dial_oracle's dense-weight functions
  // produce for that row), zero-padded to kp columns.
  void row(int64_t n, float* out, int64_t kp) const {
    switch (fmt) {
      case kW8A16: {
        const int8_t* r = q.data() + n * K;
        for (int64_t k = 0; k < K; ++k) out[k] = static_cast<float>(r[k]);
        break;
      }
      case kFp8Block128: {
        const float* t = e4m3_table().v;
        const uint8_t* r = codes.data() + n * K;
        const int64_t nbc = (K + 127) / 128;
        const float* bs = bscale.data() + (n / 128) * nbc;
        for (int64_t k = 0; k < K; ++k) out[k] = t[r[k]] * bs[k / 128];
        break;
      }
      case kNvfp4: {
        const float* t = e4m3_table().v;
        const uint8_t* r = codes.data() + n * (K / 2);
        const uint8_t* g = gscale.data() + n * (K / 16);
        for (int64_t k = 0; k < K; ++k) {
          const uint8_t c = (k & 1) ? (r[k / 2] >> 4) : (r[k / 2] & 15);
          out[k] = (kE2m1[c] * t[g[k / 16]]) * global;
        }
        break;
      }
      default: {
        const uint16_t* r = dense.data() + n * K;
        for (int64_t k = 0; k < K; ++k) out[k] = bf16_val(r[k]);
      }
    }
    for (int64_t k = K; k < kp; ++k) out[k] = 0.f;
  }
  // post-sum scale of W8A16 (applied to the f32 sum before rounding)
  float post_scale(int64_t n) const { return fmt == kW8A16 ? s[n] : 1.f; }
};

// Row-wise symmetric int8 (worker_w8a16.rs:330-341): scale = max|w| / 127
// (1.0 for a zero row), inv = 1 / scale in f32, q = clamp(round(w * inv),
// -127, 127) with round half away from zero.
void quantize_w8a16(const float* w, int64_t N, int64_t K, int8_t* q, float* s) {
#pragma omp parallel for schedule(static)
  for (int64_t n = 0; n < N; ++n) {
    const float* r = w + n * K;
    float mx = 0.f;
    for (int64_t k = 0; k < K; ++k) mx = std::max(mx, std::fabs(r[k]));
    const float sc = mx > 0.f ? mx / 127.0f : 1.0f;
    const float inv = 1.0f / sc;
    s[n] = sc;
    for (int64_t k = 0; k < K; ++k) {
      const float v = r[k] * inv;
      const double a = std::floor(std::fabs(static_cast<double>(v)) + 0.5);
      float rq = static_cast<float>(std::copysign(a, static_cast<double>(v)));
      rq = std::min(127.f, std::max(-127.f, rq));
      q[n * K + k] = static_cast<int8_t>(rq);
    }
  }
}

// Dense -> FP8 e4m3 + f32 per-128x128-block scale blockmax / 448.
void quantize_fp8_block128(const float* w, int64_t N, int64_t K, Linear& L) {
  const int64_t nbr = (N + 127) / 128, nbc = (K + 127) / 128;
  L.codes.assign(N * K, 0);
  L.bscale.assign(nbr * nbc, 1.f);
#pragma omp parallel for collapse(2) schedule(static)
  for (int64_t i = 0; i < nbr; ++i)
    for (int64_t j = 0; j < nbc; ++j) {
      const int64_t r1 = std::min(N, (i + 1) * 128), c1 = std::min(K, (j + 1) * 128);
      float am = 0.f;
      for (int64_t r = i * 128; r < r1; ++r)
        for (int64_t c = j * 128; c < c1; ++c) am = std::max(am, std::fabs(w[r * K + c]));
      const float sc = am > 0.f ? am / 448.0f : 1.0f;
      L.bscale[i * nbc + j] = sc;
      for (int64_t r = i * 128; r < r1; ++r)
        for (int64_t c = j * 128; c < c1; ++c) L.codes[r * K + c] = f32_to_e4m3(w[r * K + c] / sc);
    }
}

// Dense -> NVFP4: e2m1 in 16-element groups, e4m3 group scale of
// groupmax / 6 / global with global = amax / 6 / 448 (dial_oracle.quantize_nvfp4).
void quantize_nvfp4(const float* w, int64_t N, int64_t K, Linear& L) {
  const int64_t groups = N * K / 16;
  float amax = 0.f;
#pragma omp parallel for reduction(max : amax) schedule(static)
  for (int64_t i = 0; i < N * K; ++i) amax = std::max(amax, std::fabs(w[i]));
  const float gs = amax > 0.f ? static_cast<float>(static_cast<double>(amax) / 6.0 / 448.0) : 1.f;
  L.global = gs;
  L.codes.assign(N * K / 2, 0);
  L.gscale.assign(groups, 0);
  const float* t = e4m3_table().v;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < groups; ++g) {
    const float* v = w + g * 16;
    float gm = 0.f;
    for (int e = 0; e < 16; ++e) gm = std::max(gm, std::fabs(v[e]));
    const uint8_t sc = f32_to_e4m3(gm / 6.0f / gs);
    L.gscale[g] = sc;
    float sdec = t[sc] * gs;
    if (sdec == 0.f) sdec = 1.f;
    for (int e = 0; e < 16; e += 2)
      L.codes[g * 8 + e / 2] =
          static_cast<uint8_t>(f32_to_e2m1(v[e] / sdec) | (f32_to_e2m1(v[e + 1] / sdec) << 4));
  }
}

inline double hsum(v4d a) { return (a[0] + a[1]) + (a[2] + a[3]); }
inline float hsum(v8f a) {
  return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

// acc[c][r] = sum_k w[r][k] * x[c][k] for NR weight rows and MR activation
// rows staged in the accumulation type T (double or float), length kp (a
// multiple of 8).  Compile-time tile sizes keep the accumulators in registers.
template <class T, class V, int NR, int MR>
void micro(const T* w, int64_t kp, const T* x, int64_t xld, double acc[2][4]) {
  constexpr int L = sizeof(V) / sizeof(T);
  V a[MR][NR] = {};
  for (int64_t k = 0; k < kp; k += L) {
    V xv[MR];
#pragma GCC unroll 2
    for (int c = 0; c < MR; ++c) std::memcpy(&xv[c], x + c * xld + k, sizeof(V));
#pragma GCC unroll 4
    for (int r = 0; r < NR; ++r) {
      V wv;
      std::memcpy(&wv, w + r * kp + k, sizeof(V));
#pragma GCC unroll 2
      for (int c = 0; c < MR; ++c) a[c][r] += wv * xv[c];
    }
  }
  for (int c = 0; c < MR; ++c)
    for (int r = 0; r < NR; ++r) acc[c][r] = hsum(a[c][r]);
}

template <class T, class V>
void micro_any(const T* w, int nr, int64_t kp, const T* x, int64_t xld, int mr, double acc[2][4]) {
  switch (nr * 4 + mr) {
    case 4 * 4 + 2: micro<T, V, 4, 2>(w, kp, x, xld, acc); break;
    case 4 * 4 + 1: micro<T, V, 4, 1>(w, kp, x, xld, acc); break;
    case 3 * 4 + 2: micro<T, V, 3, 2>(w, kp, x, xld, acc); break;
    case 3 * 4 + 1: micro<T, V, 3, 1>(w, kp, x, xld, acc); break;
    case 2 * 4 + 2: micro<T, V, 2, 2>(w, kp, x, xld, acc); break;
    case 2 * 4 + 1: micro<T, V, 2, 1>(w, kp, x, xld, acc); break;
    case 1 * 4 + 2: micro<T, V, 1, 2>(w, kp, x, xld, acc); break;
    default: micro<T, V, 1, 1>(w, kp, x, xld, acc); break;
  }
}

// y[m][n] = bf16(post_scale(n) * f32(sum_k x[m][k] * W[n][k])) (+ residual
// rounding when `resid` is given: y = bf16(that + resid[m][n])).
// x holds M rows of length K (bf16 values in f32).
template <class T, class V>
void linear_forward_t(const Linear& L, const float* x, int64_t M, float* y, const float* resid) {
  const int64_t K = L.K, N = L.N, kp = (K + 7) / 8 * 8;
  std::vector<T> xp(static_cast<size_t>(M) * kp, T(0));
  for (int64_t m = 0; m < M; ++m)
    for (int64_t k = 0; k < K; ++k) xp[m * kp + k] = static_cast<T>(x[m * K + k]);
  const int64_t MB = std::max<int64_t>(2, std::min<int64_t>(M, (1 << 20) / (kp * sizeof(T)) / 2 * 2));
  for (int64_t m0 = 0; m0 < M; m0 += MB) {
    const int64_t m1 = std::min(M, m0 + MB);
#pragma omp parallel
    {
      std::vector<float> wf(kp);
      std::vector<T> wb(4 * kp);
#pragma omp for schedule(dynamic, 8)
      for (int64_t n0 = 0; n0 < N; n0 += 4) {
        const int nr = static_cast<int>(std::min<int64_t>(4, N - n0));
        for (int r = 0; r < nr; ++r) {
          L.row(n0 + r, wf.data(), kp);
          T* dst = wb.data() + r * kp;
          for (int64_t k = 0; k < kp; ++k) dst[k] = static_cast<T>(wf[k]);
        }
        for (int64_t m = m0; m < m1; m += 2) {
          const int mr = static_cast<int>(std::min<int64_t>(2, m1 - m));
          double acc[2][4];
          micro_any<T, V>(wb.data(), nr, kp, &xp[m * kp], kp, mr, acc);
          for (int c = 0; c < mr; ++c)
            for (int r = 0; r < nr; ++r) {
              const int64_t n = n0 + r;
              float v = bf16r(static_cast<float>(acc[c][r]) * L.post_scale(n));
              if (resid) v = bf16r(v + resid[(m + c) * N + n]);
              y[(m + c) * N + n] = v;
            }
        }
      }
    }
  }
}

void linear_forward(const Linear& L, const float* x, int64_t M, float* y, int accum,
                    const float* resid = nullptr) {
  if (accum == 64)
    linear_forward_t<double, v4d>(L, x, M, y, resid);
  else
    linear_forward_t<float, v8f>(L, x, M, y, resid);
}

// ------------------------------------------------------------------- norms
// candle rms_norm over rows of length n (text.rs:1466,1620-1626): sum of
// squares in f64 rounded to f32, m = bf16(sqrt(sum / n + eps)) in f32,
// y = bf16(bf16(x / m) * w).
void rms_norm_row(const float* x, const float* w, int64_t n, float eps, float* y) {
  double s2 = 0.0;
  for (int64_t i = 0; i < n; ++i) s2 += static_cast<double>(x[i]) * static_cast<double>(x[i]);
  const float sum2 = static_cast<float>(s2);
  const float m = bf16r(std::sqrt(sum2 / static_cast<float>(n) + eps));
  for (int64_t i = 0; i < n; ++i) y[i] = bf16r(bf16r(x[i] / m) * w[i]);
}

// --------------------------------------------------------------- the model
struct Cfg {
  int32_t hidden, inter, vocab, layers, heads, kv_heads;
  float eps, rope_theta;
  int32_t max_seq_len;
  int32_t fmt;  // Fmt of the layer linears
};

struct LayerW {
  Linear qkv, o, gate_up, down;
  std::vector<float> input_norm, post_norm, q_norm, k_norm;
};

struct Model {
  Cfg c{};
  int first = 0, count = 0, has_embed = 0, has_head = 0;
  int D = 128;
  std::vector<LayerW> layers;
  std::vector<uint16_t> embed;  // bf16 [vocab][hidden]
  std::vector<float> final_norm;
  Linear lm_head;  // dense bf16
  std::vector<float> cos, sin;  // bf16 values [max_seq][D/2]
  LayerW& layer(int l) { return layers[l - first]; }
};

// Per-session KV cache (cache.rs:117-237): index_pos 0 replaces, any other
// index_pos appends; keys and values per layer [kv_heads][max_seq][D].
struct Cache {
  int first = 0, kvh = 0, D = 0, max_seq = 0;
  std::vector<std::vector<float>> k, v;
  std::vector<int> len;
};

// RoPE tables (cache.rs:37-67): inv_freq = 1 / theta^(2i/d) in f32, angle =
// pos * inv_freq in f32, cos / sin of that angle rounded to bf16.
void rope_tables(Model& m) {
  const int half = m.D / 2;
  m.cos.resize(static_cast<size_t>(m.c.max_seq_len) * half);
  m.sin.resize(m.cos.size());
  for (int i = 0; i < half; ++i) {
    const float expo = static_cast<float>(2 * i) / static_cast<float>(m.D);
    const float inv = 1.0f / std::pow(m.c.rope_theta, expo);
    for (int p = 0; p < m.c.max_seq_len; ++p) {
      const float ang = static_cast<float>(p) * inv;
      m.cos[static_cast<size_t>(p) * half + i] = bf16r(static_cast<float>(std::cos(static_cast<double>(ang))));
      m.sin[static_cast<size_t>(p) * half + i] = bf16r(static_cast<float>(std::sin(static_cast<double>(ang))));
    }
  }
}

// Non-interleaved half-split rotation (text.rs:1143-1153), in place on one
// head vector of length D at position p.
void rope_vec(const Model& m, float* x, int p) {
  const int half = m.D / 2;
  const float* c = m.cos.data() + static_cast<size_t>(p) * half;
  const float* s = m.sin.data() + static_cast<size_t>(p) * half;
  for (int i = 0; i < half; ++i) {
    const float x1 = x[i], x2 = x[i + half];
    x[i] = bf16r(bf16r(x1 * c[i]) - bf16r(x2 * s[i]));
    x[i + half] = bf16r(bf16r(x1 * s[i]) + bf16r(x2 * c[i]));
  }
}

// Grouped attention for S queries of one session (text.rs:1258-1358):
// q [S][QH][D] (normed, rotated), keys / values of the layer [KVH][L][D];
// query i sits at key position L - S + i (causal when S > 1).
void attention(const Model& m, const float* q, int S, const float* kc, const float* vc, int L,
               int ldk, float* out, int round_probs) {
  const int QH = m.c.heads, KVH = m.c.kv_heads, D = m.D, rep = QH / KVH;
  const float scale = bf16r(static_cast<float>(1.0 / std::sqrt(static_cast<double>(D))));
#pragma omp parallel
  {
    std::vector<float> sc(L), e(L);
#pragma omp for collapse(2) schedule(dynamic, 1)
    for (int h = 0; h < QH; ++h)
      for (int i = 0; i < S; ++i) {
        const float* qv = q + (static_cast<size_t>(i) * QH + h) * D;
        const float* kh = kc + static_cast<size_t>(h / rep) * ldk * D;
        const float* vh = vc + static_cast<size_t>(h / rep) * ldk * D;
        const int qpos = L - S + i;
        const int jmax = S > 1 ? qpos : L - 1;
        float mx = -INFINITY;
        for (int j = 0; j <= jmax; ++j) {
          double a = 0.0;
          const float* kv = kh + static_cast<size_t>(j) * D;
          for (int d = 0; d < D; ++d) a += static_cast<double>(qv[d]) * static_cast<double>(kv[d]);
          sc[j] = bf16r(bf16r(static_cast<float>(a)) * scale);
          mx = std::max(mx, sc[j]);
        }
        double sum = 0.0;
        for (int j = 0; j <= jmax; ++j) {
          e[j] = static_cast<float>(std::exp(static_cast<double>(sc[j] - mx)));
          sum += static_cast<double>(e[j]);
        }
        const float fs = static_cast<float>(sum);
        for (int j = 0; j <= jmax; ++j) {
          const float p = e[j] / fs;
          e[j] = round_probs ? bf16r(p) : p;
        }
        float* o = out + (static_cast<size_t>(i) * QH + h) * D;
        for (int d = 0; d < D; ++d) {
          double a = 0.0;
          for (int j = 0; j <= jmax; ++j)
            a += static_cast<double>(e[j]) * static_cast<double>(vh[static_cast<size_t>(j) * D + d]);
          o[d] = bf16r(static_cast<float>(a));
        }
      }
  }
}

// Transformer::forward (text.rs:1636-1688) for one session, x [S][H] in place.
void layer_forward(Model& m, int l, Cache& cache, float* x, int S, int index_pos, int accum,
                   int round_probs) {
  LayerW& W = m.layer(l);
  const int H = m.c.hidden, I = m.c.inter, QH = m.c.heads, KVH = m.c.kv_heads, D = m.D;
  const int QKV = (QH + 2 * KVH) * D;
  std::vector<float> h(static_cast<size_t>(S) * H), qkv(static_cast<size_t>(S) * QKV);
  for (int i = 0; i < S; ++i) rms_norm_row(x + i * H, W.input_norm.data(), H, m.c.eps, &h[i * H]);
  linear_forward(W.qkv, h.data(), S, qkv.data(), accum);
  // q/k RMSNorm per head (text.rs:1466-1467,1513-1514) and RoPE
  std::vector<float> q(static_cast<size_t>(S) * QH * D);
  const int li = l - cache.first;
  std::vector<float>& kc = cache.k[li];
  std::vector<float>& vc = cache.v[li];
  const int base = index_pos == 0 ? 0 : cache.len[li];
  if (base + S > cache.max_seq) std::abort();  // callers check capacity first
  for (int i = 0; i < S; ++i) {
    const float* row = &qkv[static_cast<size_t>(i) * QKV];
    for (int hh = 0; hh < QH; ++hh) {
      float* qv = &q[(static_cast<size_t>(i) * QH + hh) * D];
      rms_norm_row(row + hh * D, W.q_norm.data(), D, m.c.eps, qv);
      rope_vec(m, qv, index_pos + i);
    }
    for (int g = 0; g < KVH; ++g) {
      float* kd = &kc[(static_cast<size_t>(g) * cache.max_seq + base + i) * D];
      float* vd = &vc[(static_cast<size_t>(g) * cache.max_seq + base + i) * D];
      rms_norm_row(row + (QH + g) * D, W.k_norm.data(), D, m.c.eps, kd);
      rope_vec(m, kd, index_pos + i);
      std::memcpy(vd, row + (QH + KVH + g) * D, D * 4);
    }
  }
  cache.len[li] = base + S;
  std::vector<float> att(static_cast<size_t>(S) * QH * D);
  attention(m, q.data(), S, kc.data(), vc.data(), base + S, cache.max_seq, att.data(), round_probs);
  // o_proj + residual, post norm, gate/up, SwiGLU, down + residual
  std::vector<float> x1(static_cast<size_t>(S) * H);
  linear_forward(W.o, att.data(), S, x1.data(), accum, x);
  for (int i = 0; i < S; ++i) rms_norm_row(&x1[i * H], W.post_norm.data(), H, m.c.eps, &h[i * H]);
  std::vector<float> gu(static_cast<size_t>(S) * 2 * I), mid(static_cast<size_t>(S) * I);
  linear_forward(W.gate_up, h.data(), S, gu.data(), accum);
  // silu(gate) * up (text.rs:816-820)
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < static_cast<int64_t>(S) * I; ++t) {
    const int64_t i = t / I, j = t % I;
    const float g = gu[i * 2 * I + j], u = gu[i * 2 * I + I + j];
    const float e = bf16r(static_cast<float>(std::exp(static_cast<double>(-g))));
    const float s = bf16r(g / bf16r(1.0f + e));
    mid[t] = bf16r(s * u);
  }
  linear_forward(W.down, mid.data(), S, x, accum, x1.data());
}

std::string g_err;

}  // namespace

// ====================================================================== C ABI
extern "C" {

typedef struct {
  int32_t hidden, inter, vocab, layers, heads, kv_heads;
  float eps, rope_theta;
  int32_t max_seq_len;
  int32_t fmt;
} orc_config;

const char* orc_last_error(void) { return g_err.c_str(); }

void orc_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}
int orc_get_threads(void) { return omp_get_max_threads(); }

void* orc_model_new(const orc_config* cfg, int first_layer, int num_layers, int has_embed,
                    int has_head) {
  auto* m = new Model();
  std::memcpy(&m->c, cfg, sizeof(Cfg));
  m->D = cfg->hidden / cfg->heads;
  m->first = first_layer;
  m->count = num_layers;
  m->has_embed = has_embed;
  m->has_head = has_head;
  m->layers.resize(num_layers);
  rope_tables(*m);
  return m;
}

void orc_model_free(void* h) { delete static_cast<Model*>(h); }

// Seeded random-init weights (dial_oracle.synth_model): bf16 N(0, std) from
// the 65536-entry quantile table, streams ((l + 1) << 8) + part for parts q,
// k, v, o, gate, up, down = 0..6, embedding 0xE0000, lm_head 0xE0002; norms
// 1.0; layer linears quantised to the model's format.
int orc_model_synth(void* h, uint64_t seed, const float* table) {
  Model& m = *static_cast<Model*>(h);
  const int64_t H = m.c.hidden, I = m.c.inter, QH = m.c.heads, KVH = m.c.kv_heads, D = m.D;
  const int64_t QKV = (QH + 2 * KVH) * D;
  std::vector<float> w(std::max({QKV * H, 2 * I * H, H * I}));
  auto st = [](int l, int p) { return (static_cast<uint64_t>(l + 1) << 8) + p; };
  auto quant = [&](Linear& L, int64_t N, int64_t K) {
    L.fmt = m.c.fmt;
    L.N = N;
    L.K = K;
    if (L.fmt == kW8A16) {
      L.q.resize(N * K);
      L.s.resize(N);
      quantize_w8a16(w.data(), N, K, L.q.data(), L.s.data());
    } else if (L.fmt == kFp8Block128) {
      quantize_fp8_block128(w.data(), N, K, L);
    } else if (L.fmt == kNvfp4) {
      quantize_nvfp4(w.data(), N, K, L);
    } else {
      L.dense.resize(N * K);
      for (int64_t i = 0; i < N * K; ++i) L.dense[i] = bf16_bits(w[i]);
    }
  };
  for (int li = 0; li < m.count; ++li) {
    const int l = m.first + li;
    LayerW& W = m.layers[li];
    synth_normal(seed, st(l, 0), QH * D * H, table, w.data());
    synth_normal(seed, st(l, 1), KVH * D * H, table, w.data() + QH * D * H);
    synth_normal(seed, st(l, 2), KVH * D * H, table, w.data() + (QH + KVH) * D * H);
    quant(W.qkv, QKV, H);
    synth_normal(seed, st(l, 3), H * QH * D, table, w.data());
    quant(W.o, H, QH * D);
    synth_normal(seed, st(l, 4), I * H, table, w.data());
    synth_normal(seed, st(l, 5), I * H, table, w.data() + I * H);
    quant(W.gate_up, 2 * I, H);
    synth_normal(seed, st(l, 6), H * I, table, w.data());
    quant(W.down, H, I);
    W.input_norm.assign(H, 1.f);
    W.post_norm.assign(H, 1.f);
    W.q_norm.assign(D, 1.f);
    W.k_norm.assign(D, 1.f);
  }
  const int64_t VH = static_cast<int64_t>(m.c.vocab) * H;
  std::vector<float>().swap(w);
  if (m.has_embed || m.has_head) {
    std::vector<float> big(VH);
    if (m.has_embed) {
      synth_normal(seed, 0xE0000, VH, table, big.data());
      m.embed.resize(VH);
#pragma omp parallel for schedule(static)
      for (int64_t i = 0; i < VH; ++i) m.embed[i] = bf16_bits(big[i]);
    }
    if (m.has_head) {
      synth_normal(seed, 0xE0002, VH, table, big.data());
      m.lm_head.fmt = kDense;
      m.lm_head.N = m.c.vocab;
      m.lm_head.K = H;
      m.lm_head.dense.resize(VH);
#pragma omp parallel for schedule(static)
      for (int64_t i = 0; i < VH; ++i) m.lm_head.dense[i] = bf16_bits(big[i]);
      m.final_norm.assign(H, 1.f);
    }
  }
  return 0;
}

// Explicit W8A16 layer weights (codes [N][K] int8, f32 row scales) and norm
// weights (bf16 values as f32); which: 0 qkv, 1 o, 2 gate_up, 3 down.
int orc_set_w8a16(void* h, int layer, int which, const int8_t* q, const float* s, int64_t N,
                  int64_t K) {
  Model& m = *static_cast<Model*>(h);
  if (layer < m.first || layer >= m.first + m.count || which < 0 || which > 3) {
    g_err = "orc_set_w8a16: bad layer or which";
    return 1;
  }
  LayerW& W = m.layer(layer);
  Linear* L[4] = {&W.qkv, &W.o, &W.gate_up, &W.down};
  L[which]->fmt = kW8A16;
  L[which]->N = N;
  L[which]->K = K;
  L[which]->q.assign(q, q + N * K);
  L[which]->s.assign(s, s + N);
  return 0;
}

// which: 0 input norm, 1 post norm, 2 q_norm, 3 k_norm.
int orc_set_norm(void* h, int layer, int which, const float* w, int64_t n) {
  Model& m = *static_cast<Model*>(h);
  if (layer < m.first || layer >= m.first + m.count || which < 0 || which > 3) {
    g_err = "orc_set_norm: bad layer or which";
    return 1;
  }
  LayerW& W = m.layer(layer);
  std::vector<float>* v[4] = {&W.input_norm, &W.post_norm, &W.q_norm, &W.k_norm};
  v[which]->assign(w, w + n);
  return 0;
}

void* orc_cache_new(void* h) {
  Model& m = *static_cast<Model*>(h);
  auto* c = new Cache();
  c->first = m.first;
  c->kvh = m.c.kv_heads;
  c->D = m.D;
  c->max_seq = m.c.max_seq_len;
  c->k.resize(m.count);
  c->v.resize(m.count);
  c->len.assign(m.count, 0);
  for (int i = 0; i < m.count; ++i) {
    c->k[i].assign(static_cast<size_t>(c->kvh) * c->max_seq * c->D, 0.f);
    c->v[i].assign(c->k[i].size(), 0.f);
  }
  return c;
}

void orc_cache_free(void* c) { delete static_cast<Cache*>(c); }

// Fill a session's cache for layers [first, first+count) with `length`
// positions of seeded bf16 values, the layout the engine's
// dial_b200_session_fill_random writes into its 16-token pages: for layer l
// the stream (l << 20) ^ (session << 4) ^ 0xCA (keys) and that + 1 (values),
// element index ((page * kv_heads + head) * 16 + token) * D + dim.
int orc_cache_fill_random(void* h, void* cp, int session, int length, uint64_t seed,
                          const float* table) {
  Model& m = *static_cast<Model*>(h);
  Cache& c = *static_cast<Cache*>(cp);
  if (length > c.max_seq) {
    g_err = "orc_cache_fill_random: length beyond capacity";
    return 1;
  }
  const int D = c.D, KVH = c.kvh;
  for (int li = 0; li < m.count; ++li) {
    const uint64_t st = (static_cast<uint64_t>(m.first + li) << 20) ^
                        (static_cast<uint64_t>(session) << 4) ^ 0xCAull;
    for (int which = 0; which < 2; ++which) {
      const uint64_t base = synth_base(seed, st + which);
      std::vector<float>& dst = which ? c.v[li] : c.k[li];
#pragma omp parallel for collapse(2) schedule(static)
      for (int g = 0; g < KVH; ++g)
        for (int t = 0; t < length; ++t) {
          const int64_t page = t / 16, tok = t % 16;
          const int64_t e0 = ((page * KVH + g) * 16 + tok) * D;
          float* o = &dst[(static_cast<size_t>(g) * c.max_seq + t) * D];
          for (int d = 0; d < D; ++d)
            o[d] = table[mix64(static_cast<uint64_t>(e0 + d) + base) & 0xffffu];
        }
    }
    c.len[li] = length;
  }
  return 0;
}

int orc_cache_len(void* cp, int layer) {
  Cache& c = *static_cast<Cache*>(cp);
  return c.len[layer - c.first];
}

// Copy out keys / values of one layer, positions [0, n): out [kv_heads][n][D].
int orc_cache_read(void* cp, int layer, int which, int n, float* out) {
  Cache& c = *static_cast<Cache*>(cp);
  const int li = layer - c.first;
  const std::vector<float>& src = which ? c.v[li] : c.k[li];
  for (int g = 0; g < c.kvh; ++g)
    std::memcpy(out + static_cast<size_t>(g) * n * c.D, &src[static_cast<size_t>(g) * c.max_seq * c.D],
                static_cast<size_t>(n) * c.D * 4);
  return 0;
}

// Embedding::forward (qwen3_vl.rs:3302): hidden [n][H] = rows of the table.
int orc_embed(void* h, const int32_t* toks, int n, float* hidden) {
  Model& m = *static_cast<Model*>(h);
  if (!m.has_embed) {
    g_err = "model has no embedding";
    return 1;
  }
  const int64_t H = m.c.hidden;
  for (int i = 0; i < n; ++i) {
    if (toks[i] < 0 || toks[i] >= m.c.vocab) {
      g_err = "token out of range";
      return 1;
    }
    for (int64_t k = 0; k < H; ++k) hidden[i * H + k] = bf16_val(m.embed[toks[i] * H + k]);
  }
  return 0;
}

// forward_blocks_from for one session: layers [first, first + count) on
// hidden [S][H] in place, starting at index_pos; capture (optional) receives
// the hidden state after each layer, [count][S][H].
int orc_forward(void* h, void* cp, float* hidden, int S, int index_pos, int first, int count,
                int accum, int round_probs, float* capture) {
  Model& m = *static_cast<Model*>(h);
  Cache& c = *static_cast<Cache*>(cp);
  if (first < m.first || first + count > m.first + m.count || S <= 0) {
    g_err = "orc_forward: layer range or row count";
    return 1;
  }
  for (int l = first; l < first + count; ++l) {
    const int base = index_pos == 0 ? 0 : c.len[l - c.first];
    if (base + S > c.max_seq || (index_pos != 0 && index_pos != base)) {
      g_err = "orc_forward: position beyond the cache capacity or not contiguous";
      return 1;
    }
  }
  const size_t HS = static_cast<size_t>(S) * m.c.hidden;
  for (int l = first; l < first + count; ++l) {
    layer_forward(m, l, c, hidden, S, index_pos, accum, round_probs);
    if (capture) std::memcpy(capture + static_cast<size_t>(l - first) * HS, hidden, HS * 4);
  }
  return 0;
}

// ln_f + dense lm_head (qwen3_vl.rs:2462-2487) on `rows` hidden rows:
// logits [rows][vocab] (bf16 values).
int orc_logits(void* h, const float* hidden, int rows, float* logits, int accum) {
  Model& m = *static_cast<Model*>(h);
  if (!m.has_head) {
    g_err = "model has no head";
    return 1;
  }
  const int64_t H = m.c.hidden;
  std::vector<float> x(static_cast<size_t>(rows) * H);
  for (int i = 0; i < rows; ++i) rms_norm_row(hidden + i * H, m.final_norm.data(), H, m.c.eps, &x[i * H]);
  linear_forward(m.lm_head, x.data(), rows, logits, accum);
  return 0;
}

// Standalone linears for the microbench parity tests: y [M][N] from x [M][K].
// fmt 0: codes int8 [N][K] + scale f32 [N]; fmt 1: e4m3 [N][K] + f32 block
// scales [ceil(N/128)][ceil(K/128)]; fmt 3: packed e2m1 [N][K/2] + e4m3
// group scales [N][K/16] + global; fmt 4: bf16 bits [N][K].
int orc_linear(int fmt, const void* codes, const void* scales, float global, int64_t N, int64_t K,
               const float* x, int64_t M, float* y, int accum) {
  Linear L;
  L.fmt = fmt;
  L.N = N;
  L.K = K;
  if (fmt == kW8A16) {
    L.q.assign(static_cast<const int8_t*>(codes), static_cast<const int8_t*>(codes) + N * K);
    L.s.assign(static_cast<const float*>(scales), static_cast<const float*>(scales) + N);
  } else if (fmt == kFp8Block128) {
    L.codes.assign(static_cast<const uint8_t*>(codes), static_cast<const uint8_t*>(codes) + N * K);
    const int64_t nb = ((N + 127) / 128) * ((K + 127) / 128);
    L.bscale.assign(static_cast<const float*>(scales), static_cast<const float*>(scales) + nb);
  } else if (fmt == kNvfp4) {
    L.codes.assign(static_cast<const uint8_t*>(codes), static_cast<const uint8_t*>(codes) + N * K / 2);
    L.gscale.assign(static_cast<const uint8_t*>(scales), static_cast<const uint8_t*>(scales) + N * K / 16);
    L.global = global;
  } else if (fmt == kDense) {
    L.dense.assign(static_cast<const uint16_t*>(codes), static_cast<const uint16_t*>(codes) + N * K);
  } else {
    g_err = "orc_linear: unknown format";
    return 1;
  }
  linear_forward(L, x, M, y, accum);
  return 0;
}

int orc_quantize_w8a16(const float* w, int64_t N, int64_t K, int8_t* q, float* s) {
  quantize_w8a16(w, N, K, q, s);
  return 0;
}

int orc_synth_normal(uint64_t seed, uint64_t stream, int64_t n, const float* table, float* out) {
  synth_normal(seed, stream, n, table, out);
  return 0;
}

// FP8 block-128 / NVFP4 quantisers of a dense [N][K] f32 weight (test weights).
int orc_quantize_fp8_block128(const float* w, int64_t N, int64_t K, uint8_t* codes, float* scales) {
  Linear L;
  quantize_fp8_block128(w, N, K, L);
  std::memcpy(codes, L.codes.data(), L.codes.size());
  std::memcpy(scales, L.bscale.data(), L.bscale.size() * 4);
  return 0;
}

int orc_quantize_nvfp4(const float* w, int64_t N, int64_t K, uint8_t* packed, uint8_t* scales,
                       float* global) {
  Linear L;
  quantize_nvfp4(w, N, K, L);
  std::memcpy(packed, L.codes.data(), L.codes.size());
  std::memcpy(scales, L.gscale.data(), L.gscale.size());
  *global = L.global;
  return 0;
}

}  // extern "C"
