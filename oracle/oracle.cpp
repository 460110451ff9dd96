// CPU ORACLE — test infrastructure only; never linked into or called by libda3b.
//
// A CPU restatement of DA3cpplib's depth hot path (preprocess -> DINOv2 backbone ->
// DPT head -> output activation), written to follow the reference's arithmetic:
// ggml CPU semantics for every graph op the reference builds (Q8_0 matmul with
// activations quantised to Q8_0 per 32-block, ggml_norm with double sums, online-
// softmax flash attention in f32, align-corners bilinear interpolation), and the
// reference's own host code for pos-embed interpolation, RoPE tables, UV embedding,
// preprocessing and output activations. Citations are path:line in DA3cpplib.
//
// Pins. The reference's own host code compiles unmodified into oracle/_ref and this
// restatement matches it bit for bit: preprocessing (src/preprocess.cpp), the UV
// embedding (src/uv_posembed.cpp), the nested alignment (src/nested.cpp), the ray ->
// pose solver (src/ray_pose.cpp, src/linalg.cpp), the 2-D RoPE tables
// (src/rope2d.cpp), the pos-embed interpolation and the multi-view reference-view
// selection (src/dino_backbone.cpp); see tests/test_oracle_pins.py and
// tests/golden/. The Q8_0 quantiser is pinned bit-exactly against gguf-py's published
// quantiser, and the DA2 architecture against an independent implementation
// (transformers). The ggml graph arithmetic (matmul, norm, flash attention, conv,
// interpolate) is a restatement only: ggml's source is absent from the reference's
// checkout (its submodule is empty) and the reference ships no golden vectors for it.
// The vectorised kernels (AVX2) keep the scalar operation order: same bits.
#include <immintrin.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <memory>
#include <string>
#include <random>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_API extern "C" __attribute__((visibility("default")))

namespace {

// ------------------------------------------------------------------ fp16
float h2f(uint16_t h) {
  const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 0x1f, m = h & 0x3ff;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = s << 31;
    } else {  // subnormal
      int ee = -1;
      uint32_t mm = m;
      do { ++ee; mm <<= 1; } while (!(mm & 0x400));
      bits = (s << 31) | ((127 - 15 - ee) << 23) | ((mm & 0x3ff) << 13);
    }
  } else if (e == 31) {
    bits = (s << 31) | 0x7f800000u | (m << 13);
  } else {
    bits = (s << 31) | ((e - 15 + 127) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
uint16_t f2h(float f) {  // round to nearest even
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000;
  const uint32_t absx = x & 0x7fffffffu;
  if (absx >= 0x7f800000u) return sign | 0x7c00 | (absx > 0x7f800000u ? 0x200 : 0);
  if (absx >= 0x477ff000u) return sign | 0x7c00;  // overflow
  if (absx < 0x38800000u) {                        // subnormal / zero
    if (absx < 0x33000000u) return sign;
    const uint32_t e = absx >> 23;
    const uint32_t m = (absx & 0x7fffff) | 0x800000;
    const int shift = 126 - e;  // 14 + (113 - e)
    const uint32_t r = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
    return sign | (r + ((rem > half) || (rem == half && (r & 1))));
  }
  const uint32_t e = (absx >> 23) - 127 + 15;
  const uint32_t m = absx & 0x7fffff;
  uint32_t h = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) ++h;
  return sign | h;
}

// Optional per-op wall-clock totals ($DA3_ORACLE_PROFILE=1 prints them after each
// forward); used to see where the checker's own time goes.
struct Prof {
  std::map<std::string, double> t;
  bool on = getenv("DA3_ORACLE_PROFILE") != nullptr;
};
Prof& prof() {
  static Prof p;
  return p;
}
struct ProfScope {
  const char* name;
  double t0;
  explicit ProfScope(const char* n) : name(n), t0(prof().on ? omp_get_wtime() : 0.0) {}
  ~ProfScope() {
    if (prof().on) prof().t[name] += omp_get_wtime() - t0;
  }
};
void prof_dump(const char* what) {
  if (!prof().on) return;
  fprintf(stderr, "[oracle %s]", what);
  for (auto& kv : prof().t) fprintf(stderr, " %s %.2fs", kv.first.c_str(), kv.second);
  fprintf(stderr, "\n");
  prof().t.clear();
}

struct Tensor {
  const void* data = nullptr;
  int type = 0;  // ggml type id: 0 f32, 1 f16, 8 q8_0
  int64_t ne[4] = {1, 1, 1, 1};
  int64_t nel() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

}  // namespace

extern "C" {
typedef struct {
  const char* name;
  const void* data;
  int type;
  int64_t ne[4];
} or_tensor;

typedef struct {
  int patch_size, embed_dim, depth, num_heads, head_dim, mlp_hidden, pos_embed_grid;
  int alt_start, rope_start, qknorm_start;
  float rope_freq, ln_eps, interp_offset;
  int cat_token, head_pos_embed, is_da2;
  int head_features;
  int n_out_layers;
  int out_layers[4];
  int head_out_channels[4];
  float img_mean[3], img_std[3];
  int resize_target, resize_upper;
  float head_max_depth;
  int act_quant;
  int n_threads;
} or_config;
}

namespace {

// ------------------------------------------------------------------ Q8_0
// ggml quantize_row_q8_0 reference: d = amax/127, id = d ? 1/d : 0, q = roundf(x*id),
// d stored as fp16 (third-party ggml, ggml-quants.c; same algorithm as gguf-py
// quants.py:378-401).
struct QBlocks {
  std::vector<float> d;     // fp16-rounded scale per block, as f32
  std::vector<int8_t> q;    // 32 per block
};

void quantize_row(const float* x, int K, float* d_out, int8_t* q_out) {
  for (int b = 0; b < K / 32; ++b) {
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(x[b * 32 + i]));
    const float d = amax / 127.0f;
    const float id = d != 0.f ? 1.0f / d : 0.0f;
    d_out[b] = h2f(f2h(d));
    for (int i = 0; i < 32; ++i) q_out[b * 32 + i] = static_cast<int8_t>(roundf(x[b * 32 + i] * id));
  }
}

// Exact int32 dot products of one 32-element int8 block of x (xb, its absolute value
// ax) with the same block of eight weight rows (w0, rows ldw bytes apart), returned as
// eight lanes. Products are formed as |x| * (w with x's sign), summed in pairs to int16
// (|q| <= 127, so no pair exceeds 32 258) and then to int32; integer sums are exact in
// any order, so each lane equals the scalar sum of x[i] * w[i].
static inline __m256i q8_dot8(__m256i xb, __m256i ax, const int8_t* w0, size_t ldw) {
  const __m256i ones = _mm256_set1_epi16(1);
  __m256i p[8];
  for (int j = 0; j < 8; ++j) {
    const __m256i wj = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(w0 + j * ldw));
    p[j] = _mm256_madd_epi16(_mm256_maddubs_epi16(ax, _mm256_sign_epi8(wj, xb)), ones);
  }
  const __m256i t0 = _mm256_hadd_epi32(p[0], p[1]), t1 = _mm256_hadd_epi32(p[2], p[3]);
  const __m256i t2 = _mm256_hadd_epi32(p[4], p[5]), t3 = _mm256_hadd_epi32(p[6], p[7]);
  const __m256i u0 = _mm256_hadd_epi32(t0, t1), u1 = _mm256_hadd_epi32(t2, t3);
  return _mm256_add_epi32(_mm256_permute2x128_si256(u0, u1, 0x20), _mm256_permute2x128_si256(u0, u1, 0x31));
}

// rows (1 or 2) activation rows (int8 qx [rows][K], scales dx [rows][K/32]) against eight
// Q8_0 weight rows (qw [8][K], scales dwT [K/32][ldd] at the first of the eight columns):
// y[r][j] = sum over blocks b in order of float(isum_b) * (d_w * d_x) (+ bias[j]), the
// scalar ggml vec_dot_q8_0_q8_0 accumulation, eight columns per vector.
static void q8_rows_x8(const int8_t* qx, const float* dx, int rows, int K, const int8_t* qw, const float* dwT,
                       int ldd, const float* bias, float* y, int ldy) {
  const int nb = K / 32;
  __m256 acc0 = _mm256_setzero_ps(), acc1 = _mm256_setzero_ps();
  for (int b = 0; b < nb; ++b) {
    const __m256 dwv = _mm256_loadu_ps(dwT + static_cast<size_t>(b) * ldd);
    const __m256i x0 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(qx + b * 32));
    const __m256i i0 = q8_dot8(x0, _mm256_sign_epi8(x0, x0), qw + b * 32, K);
    acc0 = _mm256_add_ps(acc0, _mm256_mul_ps(_mm256_cvtepi32_ps(i0), _mm256_mul_ps(dwv, _mm256_set1_ps(dx[b]))));
    if (rows > 1) {
      const __m256i x1 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(qx + K + b * 32));
      const __m256i i1 = q8_dot8(x1, _mm256_sign_epi8(x1, x1), qw + b * 32, K);
      acc1 = _mm256_add_ps(acc1,
                           _mm256_mul_ps(_mm256_cvtepi32_ps(i1), _mm256_mul_ps(dwv, _mm256_set1_ps(dx[nb + b]))));
    }
  }
  const __m256 bv = bias ? _mm256_loadu_ps(bias) : _mm256_setzero_ps();
  _mm256_storeu_ps(y, _mm256_add_ps(acc0, bv));
  if (rows > 1) _mm256_storeu_ps(y + ldy, _mm256_add_ps(acc1, bv));
}

class Oracle {
 public:
  or_config c;
  std::map<std::string, Tensor> t;
  std::map<std::string, std::vector<float>> f32cache;
  std::map<std::string, std::vector<float>> caps;  // captures for parity tests
  bool capture_resid = false;  // keep x after every block as caps["x<i>"]

  bool has(const std::string& n) const { return t.count(n) > 0; }
  const Tensor& T(const std::string& n) const {
    static Tensor empty;
    auto it = t.find(n);
    return it == t.end() ? empty : it->second;
  }
  // f32 view of an f32/f16/q8_0 tensor (converted once and cached).
  const float* F(const std::string& n) {
    auto it = t.find(n);
    if (it == t.end()) return nullptr;
    const Tensor& x = it->second;
    if (x.type == 0) return static_cast<const float*>(x.data);
    auto c2 = f32cache.find(n);
    if (c2 != f32cache.end()) return c2->second.data();
    std::vector<float> v(x.nel());
    if (x.type == 1) {
      const uint16_t* h = static_cast<const uint16_t*>(x.data);
      for (int64_t i = 0; i < x.nel(); ++i) v[i] = h2f(h[i]);
    } else if (x.type == 8) {
      const uint8_t* p = static_cast<const uint8_t*>(x.data);
      for (int64_t b = 0; b < x.nel() / 32; ++b) {
        uint16_t dh;
        memcpy(&dh, p + b * 34, 2);
        const float d = h2f(dh);
        const int8_t* q = reinterpret_cast<const int8_t*>(p + b * 34 + 2);
        for (int i = 0; i < 32; ++i) v[b * 32 + i] = d * q[i];
      }
    }
    return f32cache.emplace(n, std::move(v)).first->second.data();
  }

  // ---------------------------------------------------------------- linear
  // y[M][N] = x[M][K] W^T + b  — ggml_mul_mat(W, x) + ggml_add (src/ggml_extend.hpp:6-10).
  // Q8_0 W with act_quant: activations quantised to Q8_0, per-block int32 dot,
  // sumf += isum * (d_w * d_x) in block order (ggml vec_dot_q8_0_q8_0).
  void linear(const float* x, int M, int K, const std::string& wn, const std::string& bn, float* y) {
    ProfScope ps_("linear");
    const Tensor& W = T(wn);
    const int N = static_cast<int>(W.ne[1]);
    const float* bias = bn.empty() ? nullptr : F(bn);
    if (W.type == 8 && c.act_quant) {
      const int nb = K / 32;
      std::vector<float> dx(static_cast<size_t>(M) * nb);
      std::vector<int8_t> qx(static_cast<size_t>(M) * K);
#pragma omp parallel for schedule(static)
      for (int m = 0; m < M; ++m) quantize_row(x + static_cast<size_t>(m) * K, K, &dx[static_cast<size_t>(m) * nb], &qx[static_cast<size_t>(m) * K]);
      const uint8_t* wp = static_cast<const uint8_t*>(W.data);
      std::vector<float> dw(static_cast<size_t>(N) * nb);
      std::vector<int8_t> qw(static_cast<size_t>(N) * K);
      for (int n = 0; n < N; ++n)
        for (int b = 0; b < nb; ++b) {
          const uint8_t* blk = wp + (static_cast<size_t>(n) * nb + b) * 34;
          uint16_t dh;
          memcpy(&dh, blk, 2);
          dw[static_cast<size_t>(n) * nb + b] = h2f(dh);
          memcpy(&qw[static_cast<size_t>(n) * K + b * 32], blk + 2, 32);
        }
      // per-block scales transposed to [nb][N] so eight output columns load together
      std::vector<float> dwT(static_cast<size_t>(nb) * N);
      for (int n = 0; n < N; ++n)
        for (int b = 0; b < nb; ++b) dwT[static_cast<size_t>(b) * N + n] = dw[static_cast<size_t>(n) * nb + b];
      const int N8 = N / 8 * 8;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
      for (int n0 = 0; n0 < N8; n0 += 8)
        for (int m0 = 0; m0 < M; m0 += 64)
          for (int m = m0; m < std::min(M, m0 + 64); m += 2) {
            const int rows = std::min(2, M - m);
            q8_rows_x8(&qx[static_cast<size_t>(m) * K], &dx[static_cast<size_t>(m) * nb], rows, K,
                       &qw[static_cast<size_t>(n0) * K], &dwT[n0], N, bias ? bias + n0 : nullptr,
                       y + static_cast<size_t>(m) * N + n0, N);
          }
      // columns beyond the last multiple of 8: the same arithmetic, one column at a time
      for (int n = N8; n < N; ++n)
        for (int m = 0; m < M; ++m) {
          const int8_t* xq = &qx[static_cast<size_t>(m) * K];
          const float* xd = &dx[static_cast<size_t>(m) * nb];
          const int8_t* wq = &qw[static_cast<size_t>(n) * K];
          const float* wd = &dw[static_cast<size_t>(n) * nb];
          float sumf = 0.f;
          for (int b = 0; b < nb; ++b) {
            int isum = 0;
            for (int i = 0; i < 32; ++i) isum += static_cast<int>(wq[b * 32 + i]) * static_cast<int>(xq[b * 32 + i]);
            sumf += static_cast<float>(isum) * (wd[b] * xd[b]);
          }
          y[static_cast<size_t>(m) * N + n] = sumf + (bias ? bias[n] : 0.f);
        }
      return;
    }
    const float* w = F(wn);
    sgemm_nt(x, M, K, w, N, y);
    if (bias)
      for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) y[static_cast<size_t>(m) * N + n] += bias[n];
  }

  // y[M][N] = x[M][K] * w[N][K]^T in f32. Every output is the sum over k in order of
  // x[m][k] * w[n][k] (separate multiply and add), computed for eight columns at once
  // from w packed as [N/8][K][8].
  static void sgemm_nt(const float* x, int M, int K, const float* w, int N, float* y) {
    const int N8 = N / 8 * 8;
    std::vector<float> wp(static_cast<size_t>(N8) * K);
#pragma omp parallel for schedule(static)
    for (int nb = 0; nb < N8 / 8; ++nb)
      for (int k = 0; k < K; ++k)
        for (int j = 0; j < 8; ++j) wp[(static_cast<size_t>(nb) * K + k) * 8 + j] = w[static_cast<size_t>(nb * 8 + j) * K + k];
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int m0 = 0; m0 < M; m0 += 32)
      for (int n0 = 0; n0 < N8; n0 += 16)
        for (int m = m0; m < std::min(M, m0 + 32); m += 4) {
          const int rows = std::min(4, M - m);
          const int nv = std::min(2, (N8 - n0) / 8);
          __m256 acc[4][2];
          for (int r = 0; r < 4; ++r) acc[r][0] = acc[r][1] = _mm256_setzero_ps();
          const float* b0 = &wp[static_cast<size_t>(n0 / 8) * K * 8];
          const float* b1 = b0 + static_cast<size_t>(K) * 8;
          for (int k = 0; k < K; ++k) {
            const __m256 w0 = _mm256_loadu_ps(b0 + static_cast<size_t>(k) * 8);
            const __m256 w1 = nv > 1 ? _mm256_loadu_ps(b1 + static_cast<size_t>(k) * 8) : _mm256_setzero_ps();
            for (int r = 0; r < rows; ++r) {
              const __m256 a = _mm256_set1_ps(x[static_cast<size_t>(m + r) * K + k]);
              acc[r][0] = _mm256_add_ps(acc[r][0], _mm256_mul_ps(a, w0));
              acc[r][1] = _mm256_add_ps(acc[r][1], _mm256_mul_ps(a, w1));
            }
          }
          for (int r = 0; r < rows; ++r)
            for (int v = 0; v < nv; ++v) _mm256_storeu_ps(y + static_cast<size_t>(m + r) * N + n0 + 8 * v, acc[r][v]);
        }
    for (int n = N8; n < N; ++n)
      for (int m = 0; m < M; ++m) {
        const float* a = x + static_cast<size_t>(m) * K;
        const float* b = w + static_cast<size_t>(n) * K;
        float s2 = 0.f;
        for (int k = 0; k < K; ++k) s2 += a[k] * b[k];
        y[static_cast<size_t>(m) * N + n] = s2;
      }
  }

  // ggml_norm (double sums) * w + b  (src/ggml_extend.hpp:12-17).
  static void layernorm_rows(const float* x, int M, int D, const float* w, const float* b, float eps, float* y) {
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
      const float* r = x + static_cast<size_t>(m) * D;
      float* o = y + static_cast<size_t>(m) * D;
      double sum = 0.0;
      for (int i = 0; i < D; ++i) sum += r[i];
      const float mean = static_cast<float>(sum / D);
      double sum2 = 0.0;
      for (int i = 0; i < D; ++i) {
        const float v = r[i] - mean;
        o[i] = v;
        sum2 += static_cast<double>(v * v);
      }
      const float var = static_cast<float>(sum2 / D);
      const float scale = 1.0f / sqrtf(var + eps);
      for (int i = 0; i < D; ++i) {
        o[i] *= scale;
        o[i] = o[i] * w[i];
        if (b) o[i] += b[i];
      }
    }
  }

  // Host double-precision LayerNorm used for DA2 features (src/dino_backbone.cpp:174-181).
  static void layernorm_host(const float* row, int D, const float* w, const float* b, float eps, float* o) {
    double mean = 0;
    for (int e = 0; e < D; ++e) mean += row[e];
    mean /= D;
    double var = 0;
    for (int e = 0; e < D; ++e) {
      const double d = row[e] - mean;
      var += d * d;
    }
    var /= D;
    const double inv = 1.0 / std::sqrt(var + static_cast<double>(eps));
    for (int e = 0; e < D; ++e) o[e] = static_cast<float>((row[e] - mean) * inv) * w[e] + b[e];
  }

  // ---------------------------------------------------------------- RoPE
  // build_rope_tables (src/rope2d.cpp:4-27): head_dim split into y-half and x-half,
  // rotate-half within each half, inv_freq = freq^(-2j/half).
  struct Rope {
    std::vector<float> cos, sin;
    int hd = 0;
  };
  Rope rope_tables(const std::vector<float>& pos_yx, int tokens) const {
    Rope r;
    const int hd = c.head_dim, half = hd / 2, quart = half / 2;
    r.hd = hd;
    r.cos.assign(static_cast<size_t>(hd) * tokens, 0.f);
    r.sin.assign(static_cast<size_t>(hd) * tokens, 0.f);
    for (int tk = 0; tk < tokens; ++tk) {
      const float y = pos_yx[2 * tk], x = pos_yx[2 * tk + 1];
      for (int j = 0; j < quart; ++j) {
        const float invf = std::pow(c.rope_freq, -2.f * static_cast<float>(j) / static_cast<float>(half));
        const float ay = y * invf, ax = x * invf;
        float* cs = &r.cos[static_cast<size_t>(tk) * hd];
        float* sn = &r.sin[static_cast<size_t>(tk) * hd];
        cs[j] = cs[j + quart] = std::cos(ay);
        sn[j] = sn[j + quart] = std::sin(ay);
        cs[half + j] = cs[half + j + quart] = std::cos(ax);
        sn[half + j] = sn[half + j + quart] = std::sin(ax);
      }
    }
    return r;
  }
  // apply_rope (src/rope2d.cpp:36-52): x*cos + rot(x)*sin, rot = [-h1, h0] per half.
  static void apply_rope(float* v, const float* cs, const float* sn, int hd) {
    const int half = hd / 2, quart = half / 2;
    float rot[256];
    for (int h = 0; h < 2; ++h)
      for (int j = 0; j < quart; ++j) {
        rot[h * half + j] = -v[h * half + quart + j];
        rot[h * half + quart + j] = v[h * half + j];
      }
    for (int i = 0; i < hd; ++i) v[i] = v[i] * cs[i] + rot[i] * sn[i];
  }

  // ---------------------------------------------------------------- attention
  // attention (src/attention.cpp:44-96), flash path: per head, online softmax in f32
  // with expf, scale = 1/sqrt(head_dim) (ggml CPU flash_attn_ext with f32 K/V).
  void attention(const float* xn, int nseq, int seqlen, int blk, const Rope* rope, float* out) {
    const int D = c.embed_dim, H = c.num_heads, hd = c.head_dim;
    const int M = nseq * seqlen;
    const std::string p = "vit.blk." + std::to_string(blk) + ".";
    std::vector<float> qkv(static_cast<size_t>(M) * 3 * D);
    linear(xn, M, D, p + "attn_qkv.weight", has(p + "attn_qkv.bias") ? p + "attn_qkv.bias" : "", qkv.data());
    const bool qkn = has(p + "attn_qnorm.weight");
    const float *qw = F(p + "attn_qnorm.weight"), *qb = F(p + "attn_qnorm.bias");
    const float *kw = F(p + "attn_knorm.weight"), *kb = F(p + "attn_knorm.bias");
    // QK-norm (eps 1e-5, src/vit_block.cpp:5-11) then RoPE, per (token, head).
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
      const int tk = m % seqlen;
      for (int h = 0; h < H; ++h) {
        float* q = &qkv[static_cast<size_t>(m) * 3 * D + h * hd];
        float* k = q + D;
        if (qkn) {
          layernorm_rows(q, 1, hd, qw, qb, 1e-5f, q);
          layernorm_rows(k, 1, hd, kw, kb, 1e-5f, k);
        }
        if (rope) {
          apply_rope(q, &rope->cos[static_cast<size_t>(tk) * hd], &rope->sin[static_cast<size_t>(tk) * hd], hd);
          apply_rope(k, &rope->cos[static_cast<size_t>(tk) * hd], &rope->sin[static_cast<size_t>(tk) * hd], hd);
        }
      }
    }
    const float scale = 1.0f / std::sqrt(static_cast<float>(hd));
    std::vector<float> o(static_cast<size_t>(M) * D);
    ProfScope* ps_ = new ProfScope("attn_core");
    if (hd % 8 == 0 && hd <= 256) {
      // Keys of each (sequence, head) packed as [key block of 8][hd][8]: eight scores per
      // vector, each lane summing q[d] * k[d] over d in order like the scalar loop below.
      const int nkb = (seqlen + 7) / 8;
      std::vector<float> kt(static_cast<size_t>(nseq) * H * nkb * hd * 8, 0.f);
#pragma omp parallel for schedule(static) collapse(2)
      for (int s = 0; s < nseq; ++s)
        for (int h = 0; h < H; ++h) {
          float* dst = &kt[(static_cast<size_t>(s) * H + h) * nkb * hd * 8];
          for (int ki = 0; ki < seqlen; ++ki) {
            const float* k = &qkv[(static_cast<size_t>(s) * seqlen + ki) * 3 * D + D + h * hd];
            for (int d = 0; d < hd; ++d) dst[(static_cast<size_t>(ki / 8) * hd + d) * 8 + (ki % 8)] = k[d];
          }
        }
      const int nv = hd / 8;
      // two queries of one (sequence, head) at a time: independent online-softmax chains
      // interleaved, sharing the key and value loads; each query's arithmetic and order are
      // those of the scalar loop below
      const int nqp = (seqlen + 1) / 2;
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
      for (int s = 0; s < nseq; ++s)
        for (int qp = 0; qp < nqp; ++qp)
          for (int h = 0; h < H; ++h) {
            const int nq = std::min(2, seqlen - 2 * qp);
            const float* q[2];
            for (int r = 0; r < 2; ++r)
              q[r] = &qkv[(static_cast<size_t>(s) * seqlen + 2 * qp + std::min(r, nq - 1)) * 3 * D + h * hd];
            const float* kth = &kt[(static_cast<size_t>(s) * H + h) * nkb * hd * 8];
            __m256 acc[2][32];
            for (int r = 0; r < 2; ++r)
              for (int v = 0; v < nv; ++v) acc[r][v] = _mm256_setzero_ps();
            float Mx[2] = {-INFINITY, -INFINITY}, S[2] = {0.f, 0.f};
            alignas(32) float sc8[2][8];
            for (int kb = 0; kb < nkb; ++kb) {
              const float* kp = kth + static_cast<size_t>(kb) * hd * 8;
              __m256 dot0 = _mm256_setzero_ps(), dot1 = _mm256_setzero_ps();
              for (int d = 0; d < hd; ++d) {
                const __m256 kv = _mm256_loadu_ps(kp + d * 8);
                dot0 = _mm256_add_ps(dot0, _mm256_mul_ps(_mm256_set1_ps(q[0][d]), kv));
                dot1 = _mm256_add_ps(dot1, _mm256_mul_ps(_mm256_set1_ps(q[1][d]), kv));
              }
              _mm256_store_ps(sc8[0], _mm256_mul_ps(dot0, _mm256_set1_ps(scale)));
              _mm256_store_ps(sc8[1], _mm256_mul_ps(dot1, _mm256_set1_ps(scale)));
              const int nk = std::min(8, seqlen - kb * 8);
              for (int j = 0; j < nk; ++j) {
                const float* vrow = &qkv[(static_cast<size_t>(s) * seqlen + kb * 8 + j) * 3 * D + 2 * D + h * hd];
                for (int r = 0; r < 2; ++r) {
                  const float sc = sc8[r][j];
                  float ms = 1.f, vs = 1.f;
                  if (sc > Mx[r]) {
                    const float Mold = Mx[r];
                    Mx[r] = sc;
                    ms = expf(Mold - Mx[r]);
                    const __m256 msv = _mm256_set1_ps(ms);
                    for (int v = 0; v < nv; ++v) acc[r][v] = _mm256_mul_ps(acc[r][v], msv);
                  } else {
                    vs = expf(sc - Mx[r]);
                  }
                  const __m256 vsv = _mm256_set1_ps(vs);
                  for (int v = 0; v < nv; ++v)
                    acc[r][v] = _mm256_add_ps(acc[r][v], _mm256_mul_ps(_mm256_loadu_ps(vrow + 8 * v), vsv));
                  S[r] = S[r] * ms + vs;
                }
              }
            }
            for (int r = 0; r < nq; ++r) {
              float* od = &o[(static_cast<size_t>(s) * seqlen + 2 * qp + r) * D + h * hd];
              const float inv = S[r] == 0.f ? 0.f : 1.0f / S[r];
              const __m256 iv = _mm256_set1_ps(inv);
              for (int v = 0; v < nv; ++v) _mm256_storeu_ps(od + 8 * v, _mm256_mul_ps(acc[r][v], iv));
            }
          }
      delete ps_;
      linear(o.data(), M, D, p + "attn_proj.weight", has(p + "attn_proj.bias") ? p + "attn_proj.bias" : "", out);
      return;
    }
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
    for (int s = 0; s < nseq; ++s)
      for (int qi = 0; qi < seqlen; ++qi)
        for (int h = 0; h < H; ++h) {
          const float* q = &qkv[(static_cast<size_t>(s) * seqlen + qi) * 3 * D + h * hd];
          float acc[256];
          for (int d = 0; d < hd; ++d) acc[d] = 0.f;
          float Mx = -INFINITY, S = 0.f;
          for (int ki = 0; ki < seqlen; ++ki) {
            const float* k = &qkv[(static_cast<size_t>(s) * seqlen + ki) * 3 * D + D + h * hd];
            const float* v = k + D;
            float sc = 0.f;
            for (int d = 0; d < hd; ++d) sc += q[d] * k[d];
            sc *= scale;
            float ms = 1.f, vs = 1.f;
            if (sc > Mx) {
              const float Mold = Mx;
              Mx = sc;
              ms = expf(Mold - Mx);
              for (int d = 0; d < hd; ++d) acc[d] *= ms;
            } else {
              vs = expf(sc - Mx);
            }
            for (int d = 0; d < hd; ++d) acc[d] += v[d] * vs;
            S = S * ms + vs;
          }
          float* od = &o[(static_cast<size_t>(s) * seqlen + qi) * D + h * hd];
          const float inv = S == 0.f ? 0.f : 1.0f / S;
          for (int d = 0; d < hd; ++d) od[d] = acc[d] * inv;
        }
    delete ps_;
    linear(o.data(), M, D, p + "attn_proj.weight", has(p + "attn_proj.bias") ? p + "attn_proj.bias" : "", out);
  }

  // vit_block (src/vit_block.cpp:30-58): x += ls1*Attn(LN1 x); x += ls2*fc2(gelu(fc1(LN2 x))).
  void vit_block(float* x, int nseq, int seqlen, int blk, const Rope* rope) {
    const int D = c.embed_dim, M = nseq * seqlen, Hm = c.mlp_hidden;
    const std::string p = "vit.blk." + std::to_string(blk) + ".";
    std::vector<float> xn(static_cast<size_t>(M) * D), a(static_cast<size_t>(M) * D);
    layernorm_rows(x, M, D, F(p + "norm1.weight"), F(p + "norm1.bias"), c.ln_eps, xn.data());
    attention(xn.data(), nseq, seqlen, blk, rope, a.data());
    const float* ls1 = F(p + "ls1");
    for (size_t i = 0; i < a.size(); ++i) x[i] += ls1 ? a[i] * ls1[i % D] : a[i];
    layernorm_rows(x, M, D, F(p + "norm2.weight"), F(p + "norm2.bias"), c.ln_eps, xn.data());
    std::vector<float> h(static_cast<size_t>(M) * Hm);
    linear(xn.data(), M, D, p + "mlp_fc1.weight", p + "mlp_fc1.bias", h.data());
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < h.size(); ++i) h[i] = 0.5f * h[i] * (1.0f + erff(h[i] * 0.70710678118654752440f));
    linear(h.data(), M, Hm, p + "mlp_fc2.weight", p + "mlp_fc2.bias", a.data());
    const float* ls2 = F(p + "ls2");
    for (size_t i = 0; i < a.size(); ++i) x[i] += ls2 ? a[i] * ls2[i % D] : a[i];
  }

  // ---------------------------------------------------------------- embeddings
  static float cubic(float x) {  // a = -0.75 (src/dino_backbone.cpp:12-17)
    const float a = -0.75f;
    x = std::fabs(x);
    if (x < 1) return ((a + 2) * x - (a + 3)) * x * x + 1;
    if (x < 2) return (((x - 5) * x + 8) * x - 4) * a;
    return 0;
  }
  // interp_pos_embed (src/dino_backbone.cpp:18-56): always bicubic with the offset.
  std::vector<float> interp_pos_embed(int gh, int gw) {
    const int E = c.embed_dim, Mg = c.pos_embed_grid;
    const float* p = F("vit.pos_embed");
    std::vector<float> out(static_cast<size_t>(1 + gh * gw) * E);
    for (int ch = 0; ch < E; ++ch) out[ch] = p[ch];
    const float sx = static_cast<float>(gw + c.interp_offset) / Mg, sy = static_cast<float>(gh + c.interp_offset) / Mg;
    for (int oy = 0; oy < gh; ++oy) {
      const float iy = (oy + 0.5f) / sy - 0.5f;
      const int y0 = static_cast<int>(std::floor(iy));
      const float fy = iy - y0;
      for (int ox = 0; ox < gw; ++ox) {
        const float ix = (ox + 0.5f) / sx - 0.5f;
        const int x0 = static_cast<int>(std::floor(ix));
        const float fx = ix - x0;
        const int orow = 1 + oy * gw + ox;
        for (int ch = 0; ch < E; ++ch) {
          float acc = 0;
          for (int m = -1; m <= 2; ++m) {
            const float wy = cubic(fy - m);
            const int yy = std::min(std::max(y0 + m, 0), Mg - 1);
            for (int n = -1; n <= 2; ++n) {
              const float wx = cubic(fx - n);
              const int xx = std::min(std::max(x0 + n, 0), Mg - 1);
              acc += wy * wx * p[static_cast<size_t>(1 + yy * Mg + xx) * E + ch];
            }
          }
          out[static_cast<size_t>(orow) * E + ch] = acc;
        }
      }
    }
    return out;
  }

  // Patch embed conv k14 s14 + bias, CLS concat, + pos-embed (src/dino_backbone.cpp:117-126).
  void embed(const float* chw, int H, int W, const std::vector<float>& pos, float* x) {
    const int P = c.patch_size, E = c.embed_dim, gh = H / P, gw = W / P;
    const float* pw = F("vit.patch_embed.weight");  // [E][3][P][P]
    const float* pb = F("vit.patch_embed.bias");
    const float* cls = F("vit.cls_token");
    for (int e = 0; e < E; ++e) x[e] = cls[e] + pos[e];
#pragma omp parallel for schedule(static)
    for (int t = 0; t < gh * gw; ++t) {
      const int py = t / gw, px = t % gw;
      for (int e = 0; e < E; ++e) {
        float s = 0.f;
        for (int ch = 0; ch < 3; ++ch)
          for (int ky = 0; ky < P; ++ky) {
            const float* img = chw + (static_cast<size_t>(ch) * H + py * P + ky) * W + px * P;
            const float* w = pw + ((static_cast<size_t>(e) * 3 + ch) * P + ky) * P;
            for (int kx = 0; kx < P; ++kx) s += w[kx] * img[kx];
          }
        x[static_cast<size_t>(1 + t) * E + e] = s + pb[e] + pos[static_cast<size_t>(1 + t) * E + e];
      }
    }
  }

  // ---------------------------------------------------------------- head ops (NCHW per image)
  struct Map {
    int C = 0, H = 0, W = 0;
    std::vector<float> v;  // [C][H][W]
    Map() {}
    Map(int c_, int h_, int w_) : C(c_), H(h_), W(w_), v(static_cast<size_t>(c_) * h_ * w_, 0.f) {}
    float* ch(int cc) { return &v[static_cast<size_t>(cc) * H * W]; }
    const float* ch(int cc) const { return &v[static_cast<size_t>(cc) * H * W]; }
  };

  // conv2d with ggml kernel [KW,KH,IC,OC] (= torch [OC][IC][KH][KW]) f32, stride s, pad p,
  // optional bias (src/dpt_blocks.cpp:18-66, direct f32 semantics).
  Map conv2d(const Map& x, const std::string& wn, const std::string& bn, int stride, int pad) {
    ProfScope ps_("conv2d");
    const Tensor& Wt = T(wn);
    const int ks = static_cast<int>(Wt.ne[0]), IC = static_cast<int>(Wt.ne[2]), OC = static_cast<int>(Wt.ne[3]);
    const float* w = F(wn);
    const float* b = (!bn.empty() && has(bn)) ? F(bn) : nullptr;
    const int Ho = (x.H + 2 * pad - ks) / stride + 1, Wo = (x.W + 2 * pad - ks) / stride + 1;
    Map y(OC, Ho, Wo);
    // Sixteen output channels per pair of vectors: weights packed [oc/16][ic][tap][16]
    // (zero beyond OC), each output pixel's sixteen sums held in registers while its
    // terms are added in the order ic, ky, kx (taps outside the input are skipped, as a
    // direct convolution does), then the bias. Interior pixels go four at a time.
    const int KK = ks * ks, nob = (OC + 15) / 16;
    std::vector<float> wp(static_cast<size_t>(nob) * IC * KK * 16, 0.f);
    for (int oc = 0; oc < OC; ++oc)
      for (int ic = 0; ic < IC; ++ic)
        for (int t = 0; t < KK; ++t)
          wp[((static_cast<size_t>(oc / 16) * IC + ic) * KK + t) * 16 + oc % 16] =
              w[(static_cast<size_t>(oc) * IC + ic) * KK + t];
    const size_t plane = static_cast<size_t>(x.H) * x.W;
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int ob = 0; ob < nob; ++ob)
      for (int oy = 0; oy < Ho; ++oy) {
        const float* wb = &wp[static_cast<size_t>(ob) * IC * KK * 16];
        const int nlane = std::min(16, OC - ob * 16);
        auto store = [&](int ox, __m256 lo, __m256 hi) {
          alignas(32) float v[16];
          _mm256_store_ps(v, lo);
          _mm256_store_ps(v + 8, hi);
          for (int j = 0; j < nlane; ++j) {
            const int oc = ob * 16 + j;
            y.v[(static_cast<size_t>(oc) * Ho + oy) * Wo + ox] = b ? v[j] + b[oc] : v[j];
          }
        };
        const int iy0 = oy * stride - pad;
        const bool rows_in = iy0 >= 0 && iy0 + ks <= x.H;
        int ox = 0;
        if (rows_in) {
          // interior run: every tap of pixels ox..ox+3 inside the input
          const int lo = (pad + stride - 1) / stride;  // first ox whose leftmost tap is >= 0
          const int hi = (x.W - ks + pad) / stride;    // last ox whose rightmost tap is < W
          for (; ox < Wo && ox < lo; ++ox) {
            __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
            conv_pixel(x, wb, IC, ks, stride, pad, oy, ox, plane, a0, a1);
            store(ox, a0, a1);
          }
          for (; ox + 3 <= hi && ox + 3 < Wo; ox += 4) {
            __m256 a[4][2];
            for (int r = 0; r < 4; ++r) a[r][0] = a[r][1] = _mm256_setzero_ps();
            const int ix0 = ox * stride - pad;
            for (int ic = 0; ic < IC; ++ic) {
              const float* in = x.v.data() + ic * plane;
              for (int ky = 0; ky < ks; ++ky) {
                const float* row = in + static_cast<size_t>(iy0 + ky) * x.W + ix0;
                for (int kx = 0; kx < ks; ++kx) {
                  const float* wt = wb + (static_cast<size_t>(ic) * KK + ky * ks + kx) * 16;
                  const __m256 w0 = _mm256_loadu_ps(wt), w1 = _mm256_loadu_ps(wt + 8);
                  for (int r = 0; r < 4; ++r) {
                    const __m256 v = _mm256_set1_ps(row[r * stride + kx]);
                    a[r][0] = _mm256_add_ps(a[r][0], _mm256_mul_ps(v, w0));
                    a[r][1] = _mm256_add_ps(a[r][1], _mm256_mul_ps(v, w1));
                  }
                }
              }
            }
            for (int r = 0; r < 4; ++r) store(ox + r, a[r][0], a[r][1]);
          }
        }
        for (; ox < Wo; ++ox) {
          __m256 a0 = _mm256_setzero_ps(), a1 = _mm256_setzero_ps();
          conv_pixel(x, wb, IC, ks, stride, pad, oy, ox, plane, a0, a1);
          store(ox, a0, a1);
        }
      }
    return y;
  }

  // One output pixel of conv2d (sixteen output channels), skipping taps outside the input.
  static void conv_pixel(const Map& x, const float* wb, int IC, int ks, int stride, int pad, int oy, int ox,
                         size_t plane, __m256& a0, __m256& a1) {
    const int KK = ks * ks;
    for (int ic = 0; ic < IC; ++ic) {
      const float* in = x.v.data() + ic * plane;
      for (int ky = 0; ky < ks; ++ky) {
        const int iy = oy * stride + ky - pad;
        if (iy < 0 || iy >= x.H) continue;
        for (int kx = 0; kx < ks; ++kx) {
          const int ix = ox * stride + kx - pad;
          if (ix < 0 || ix >= x.W) continue;
          const float* wt = wb + (static_cast<size_t>(ic) * KK + ky * ks + kx) * 16;
          const __m256 v = _mm256_set1_ps(in[static_cast<size_t>(iy) * x.W + ix]);
          a0 = _mm256_add_ps(a0, _mm256_mul_ps(v, _mm256_loadu_ps(wt)));
          a1 = _mm256_add_ps(a1, _mm256_mul_ps(v, _mm256_loadu_ps(wt + 8)));
        }
      }
    }
  }

  // conv_transpose2d_p0 with stride == kernel; ggml kernel [KW,KH,OC,IC]
  // (= torch [IC][OC][KH][KW]) (src/dpt_blocks.cpp:68-85).
  Map convT(const Map& x, const std::string& wn, const std::string& bn, int S) {
    ProfScope ps_("convT");
    const Tensor& Wt = T(wn);
    const int OC = static_cast<int>(Wt.ne[2]), IC = static_cast<int>(Wt.ne[3]);
    const float* w = F(wn);
    const float* b = has(bn) ? F(bn) : nullptr;
    Map y(OC, x.H * S, x.W * S);
#pragma omp parallel for schedule(dynamic, 1)
    for (int oc = 0; oc < OC; ++oc)
      for (int ky = 0; ky < S; ++ky)
        for (int kx = 0; kx < S; ++kx) {
          float* out = y.ch(oc);
          for (int iy = 0; iy < x.H; ++iy)
            for (int ix = 0; ix < x.W; ++ix) out[static_cast<size_t>(iy * S + ky) * y.W + ix * S + kx] = b ? b[oc] : 0.f;
          for (int ic = 0; ic < IC; ++ic) {
            const float wv = w[((static_cast<size_t>(ic) * OC + oc) * S + ky) * S + kx];
            const float* in = x.ch(ic);
            for (int iy = 0; iy < x.H; ++iy)
              for (int ix = 0; ix < x.W; ++ix)
                out[static_cast<size_t>(iy * S + ky) * y.W + ix * S + kx] += wv * in[static_cast<size_t>(iy) * x.W + ix];
          }
        }
    return y;
  }

  // ggml_interpolate bilinear + align corners (src/dpt_blocks.cpp:87-90): ggml CPU
  // upscale with pixel_offset 0 and sf = (dst-1)/(src-1), y = i / sf.
  static Map interp_ac(const Map& x, int ow, int oh) {
    Map y(x.C, oh, ow);
    const float sf0 = (ow > 1 && x.W > 1) ? static_cast<float>(ow - 1) / (x.W - 1) : static_cast<float>(ow) / x.W;
    const float sf1 = (oh > 1 && x.H > 1) ? static_cast<float>(oh - 1) / (x.H - 1) : static_cast<float>(oh) / x.H;
#pragma omp parallel for schedule(static)
    for (int cc = 0; cc < x.C; ++cc) {
      const float* in = x.ch(cc);
      float* out = y.ch(cc);
      for (int i1 = 0; i1 < oh; ++i1) {
        const float fy = static_cast<float>(i1) / sf1;
        int64_t y0 = static_cast<int64_t>(floorf(fy)), y1 = y0 + 1;
        y0 = std::max<int64_t>(0, std::min<int64_t>(y0, x.H - 1));
        y1 = std::max<int64_t>(0, std::min<int64_t>(y1, x.H - 1));
        float dy = fy - floorf(fy);
        dy = std::max(0.0f, std::min(dy, 1.0f));
        for (int i0 = 0; i0 < ow; ++i0) {
          const float fx = static_cast<float>(i0) / sf0;
          int64_t x0 = static_cast<int64_t>(floorf(fx)), x1 = x0 + 1;
          x0 = std::max<int64_t>(0, std::min<int64_t>(x0, x.W - 1));
          x1 = std::max<int64_t>(0, std::min<int64_t>(x1, x.W - 1));
          float dx = fx - floorf(fx);
          dx = std::max(0.0f, std::min(dx, 1.0f));
          const float a = in[y0 * x.W + x0], b = in[y0 * x.W + x1], cc2 = in[y1 * x.W + x0], d = in[y1 * x.W + x1];
          out[static_cast<size_t>(i1) * ow + i0] =
              a * (1 - dx) * (1 - dy) + b * dx * (1 - dy) + cc2 * (1 - dx) * dy + d * dx * dy;
        }
      }
    }
    return y;
  }

  static void relu_inplace(Map& m) {
    for (auto& v : m.v) v = std::max(v, 0.0f);
  }
  static void add_inplace(Map& a, const Map& b) {
    for (size_t i = 0; i < a.v.size(); ++i) a.v[i] += b.v[i];
  }

  // residual_conv_unit (src/dpt_blocks.cpp:92-114).
  Map rcu(const Map& x, const std::string& p) {
    Map o = x;
    relu_inplace(o);
    o = conv2d(o, p + "c1.weight", p + "c1.bias", 1, 1);
    relu_inplace(o);
    o = conv2d(o, p + "c2.weight", p + "c2.bias", 1, 1);
    add_inplace(o, x);
    return o;
  }
  // feature_fusion (src/dpt_blocks.cpp:116-143).
  Map fusion(const Map& top, const Map* lateral, const std::string& p, int ow, int oh) {
    Map y = top;
    if (lateral && has(p + "rc1.c1.weight")) {
      Map r = rcu(*lateral, p + "rc1.");
      add_inplace(y, r);
    }
    y = rcu(y, p + "rc2.");
    const int w2 = ow > 0 ? ow : y.W * 2, h2 = oh > 0 ? oh : y.H * 2;
    y = interp_ac(y, w2, h2);
    return conv2d(y, p + "out.weight", p + "out.bias", 1, 0);
  }

  // uv_pos_embed (src/uv_posembed.cpp:15-73) * ratio, as [C][H][W].
  static Map uv_embed(int pw, int ph, int C, float aspect, float ratio) {
    Map m(C, ph, pw);
    const double diag = std::sqrt(static_cast<double>(aspect) * aspect + 1.0);
    const double span_x = aspect / diag, span_y = 1.0 / diag;
    const double left_x = -span_x * (pw - 1) / pw, right_x = span_x * (pw - 1) / pw;
    const double top_y = -span_y * (ph - 1) / ph, bottom_y = span_y * (ph - 1) / ph;
    std::vector<double> xc(pw), yc(ph);
    for (int i = 0; i < pw; ++i) xc[i] = pw == 1 ? left_x : left_x + i * ((right_x - left_x) / (pw - 1));
    for (int i = 0; i < ph; ++i) yc[i] = ph == 1 ? top_y : top_y + i * ((bottom_y - top_y) / (ph - 1));
    const int D = C / 2, Fq = D / 2;
    std::vector<double> om(Fq);
    for (int j = 0; j < Fq; ++j) om[j] = 1.0 / std::pow(100.0, static_cast<double>(j) / (static_cast<double>(D) / 2.0));
    for (int y = 0; y < ph; ++y)
      for (int x = 0; x < pw; ++x)
        for (int j = 0; j < Fq; ++j) {
          const double ox = xc[x] * om[j], oy = yc[y] * om[j];
          const size_t pix = static_cast<size_t>(y) * pw + x, hw = static_cast<size_t>(pw) * ph;
          m.v[(j)*hw + pix] = ratio * static_cast<float>(std::sin(ox));
          m.v[(Fq + j) * hw + pix] = ratio * static_cast<float>(std::cos(ox));
          m.v[(D + j) * hw + pix] = ratio * static_cast<float>(std::sin(oy));
          m.v[(D + Fq + j) * hw + pix] = ratio * static_cast<float>(std::cos(oy));
        }
    return m;
  }

  // DptHead::build_depth_graph (src/dpt_head.cpp:75-275) for one image. feats[s]:
  // [Npatch][C] token-major. Returns main logits [od][H][W]; aux logits [7][Ha][Wa]
  // when the aux tensors exist and want_aux.
  // sky_out (when non-null and the sky tensors exist) receives the sky logits [1][H][W]
  // of the metric / mono DPT (src/dpt_head.cpp:205-222).
  Map head(const std::vector<const float*>& feats, int Cf, int H, int W, bool want_aux, Map* aux_out, const std::string& cap,
           Map* sky_out = nullptr) {
    const int P = c.patch_size, pw = W / P, ph = H / P, N = pw * ph;
    const float aspect = static_cast<float>(W) / H;
    const bool hn = has("head.norm.weight");
    Map l[4];
    for (int s = 0; s < 4; ++s) {
      std::vector<float> f(feats[s], feats[s] + static_cast<size_t>(N) * Cf);
      if (hn) layernorm_rows(f.data(), N, Cf, F("head.norm.weight"), F("head.norm.bias"), 1e-5f, f.data());
      Map x(Cf, ph, pw);
      for (int tk = 0; tk < N; ++tk)
        for (int ch = 0; ch < Cf; ++ch) x.v[static_cast<size_t>(ch) * N + tk] = f[static_cast<size_t>(tk) * Cf + ch];
      const std::string ss = std::to_string(s);
      x = conv2d(x, "head.proj." + ss + ".weight", "head.proj." + ss + ".bias", 1, 0);
      if (c.head_pos_embed) add_inplace(x, uv_embed(pw, ph, x.C, aspect, 0.1f));
      if (s == 0) x = convT(x, "head.resize.0.weight", "head.resize.0.bias", 4);
      else if (s == 1) x = convT(x, "head.resize.1.weight", "head.resize.1.bias", 2);
      else if (s == 3) x = conv2d(x, "head.resize.3.weight", "head.resize.3.bias", 2, 1);
      l[s] = std::move(x);
      caps[cap + "stage" + ss] = l[s].v;
    }
    Map rn[4];
    for (int s = 0; s < 4; ++s) rn[s] = conv2d(l[s], "head.scratch.layer" + std::to_string(s + 1) + "_rn.weight", "", 1, 1);
    auto pyramid = [&](const std::string& sfx) {
      Map o = fusion(rn[3], nullptr, "head.scratch.rn4" + sfx + ".", pw, ph);
      o = fusion(o, &rn[2], "head.scratch.rn3" + sfx + ".", 2 * pw, 2 * ph);
      o = fusion(o, &rn[1], "head.scratch.rn2" + sfx + ".", 4 * pw, 4 * ph);
      o = fusion(o, &rn[0], "head.scratch.rn1" + sfx + ".", 0, 0);
      return o;
    };
    Map out = pyramid("");
    out = conv2d(out, "head.scratch.out1.weight", "head.scratch.out1.bias", 1, 1);
    caps[cap + "out1"] = out.v;
    out = interp_ac(out, W, H);
    if (c.head_pos_embed) add_inplace(out, uv_embed(W, H, out.C, aspect, 0.1f));
    if (sky_out && has("head.scratch.sky_out2b.weight")) {
      Map sk = conv2d(out, "head.scratch.sky_out2a.weight", "head.scratch.sky_out2a.bias", 1, 1);
      relu_inplace(sk);
      *sky_out = conv2d(sk, "head.scratch.sky_out2b.weight", "head.scratch.sky_out2b.bias", 1, 0);
    }
    out = conv2d(out, "head.scratch.out2a.weight", "head.scratch.out2a.bias", 1, 1);
    relu_inplace(out);
    out = conv2d(out, "head.scratch.out2b.weight", "head.scratch.out2b.bias", 1, 0);
    if (want_aux && aux_out && has("head.scratch.rn1_aux.out.weight")) {
      Map a = pyramid("_aux");
      for (int i = 0; i < 5; ++i) {
        const std::string p = "head.scratch.out1_aux." + std::to_string(i) + ".";
        a = conv2d(a, p + "weight", p + "bias", 1, 1);
      }
      if (c.head_pos_embed) add_inplace(a, uv_embed(a.W, a.H, a.C, aspect, 0.1f));
      a = conv2d(a, "head.scratch.out2a_aux.weight", "head.scratch.out2a_aux.bias", 1, 1);
      // channels-last LayerNorm over C (eps 1e-5) (src/dpt_head.cpp:56-66, :268-269)
      {
        const float* g = F("head.scratch.out2_aux_ln.weight");
        const float* b = F("head.scratch.out2_aux_ln.bias");
        const int HW = a.H * a.W;
        std::vector<float> px(a.C);
        for (int p = 0; p < HW; ++p) {
          for (int ch = 0; ch < a.C; ++ch) px[ch] = a.v[static_cast<size_t>(ch) * HW + p];
          layernorm_rows(px.data(), 1, a.C, g, b, 1e-5f, px.data());
          for (int ch = 0; ch < a.C; ++ch) a.v[static_cast<size_t>(ch) * HW + p] = px[ch];
        }
      }
      relu_inplace(a);
      a = conv2d(a, "head.scratch.out2b_aux.weight", "head.scratch.out2b_aux.bias", 1, 0);
      *aux_out = std::move(a);
    }
    return out;
  }

  // ---------------------------------------------------------------- backbone
  // Positions (src/dino_backbone.cpp:92-95): token 0 at (0,0); patch t: local (row+1, col+1),
  // nodiff (1,1).
  void positions(int gh, int gw, std::vector<float>& local, std::vector<float>& nodiff) const {
    const int Nt = 1 + gh * gw;
    local.assign(2 * Nt, 0.f);
    nodiff.assign(2 * Nt, 0.f);
    for (int tk = 1; tk < Nt; ++tk) {
      const int idx = tk - 1, row = idx / gw, col = idx % gw;
      local[2 * tk] = static_cast<float>(row + 1);
      local[2 * tk + 1] = static_cast<float>(col + 1);
      nodiff[2 * tk] = nodiff[2 * tk + 1] = 1.f;
    }
  }

  // Multi-view backbone (S >= 1 views already in processing order), returning per
  // out-layer features [S][Npatch][C] (src/dino_backbone.cpp:80-213, 462-616).
  // upto >= 0 stops after block upto-1 and returns x (pass A helper).
  void backbone(const std::vector<std::vector<float>>& views, int H, int W, std::vector<std::vector<float>>& feats,
                int upto, std::vector<float>* x_out, std::vector<std::vector<float>>* cams = nullptr) {
    const int P = c.patch_size, gh = H / P, gw = W / P, Np = gh * gw, Nt = 1 + Np, E = c.embed_dim;
    const int S = static_cast<int>(views.size());
    std::vector<float> pos = interp_pos_embed(gh, gw);
    std::vector<float> x(static_cast<size_t>(S) * Nt * E);
    for (int s = 0; s < S; ++s) embed(views[s].data(), H, W, pos, &x[static_cast<size_t>(s) * Nt * E]);
    std::vector<float> pl, pn;
    positions(gh, gw, pl, pn);
    Rope r_local = rope_tables(pl, Nt);
    std::vector<float> png(2 * static_cast<size_t>(Nt) * S);
    for (int s = 0; s < S; ++s)
      for (int tk = 0; tk < Nt; ++tk) {
        png[2 * (static_cast<size_t>(s) * Nt + tk)] = pn[2 * tk];
        png[2 * (static_cast<size_t>(s) * Nt + tk) + 1] = pn[2 * tk + 1];
      }
    Rope r_global = rope_tables(png, Nt * S);
    const float* cam = F("vit.camera_token");
    std::vector<float> local_x = x;
    const int NL = c.n_out_layers;
    feats.assign(NL, std::vector<float>());
    if (cams) cams->assign(NL, std::vector<float>());
    const int depth = upto >= 0 ? upto : c.depth;
    for (int i = 0; i < depth; ++i) {
      if (c.alt_start >= 0 && i == c.alt_start) {
        for (int s = 0; s < S; ++s)  // token 0 <- camera_token[ref slot 0 | src slot 1]
          for (int e = 0; e < E; ++e) x[static_cast<size_t>(s) * Nt * E + e] = cam ? cam[(s == 0 ? 0 : E) + e] : 0.f;
      }
      const bool global = c.alt_start >= 0 && i >= c.alt_start && (i % 2 == 1);
      const bool use_rope = c.rope_start >= 0 && i >= c.rope_start;
      if (global) vit_block(x.data(), 1, S * Nt, i, use_rope ? &r_global : nullptr);
      else vit_block(x.data(), S, Nt, i, use_rope ? &r_local : nullptr);
      if (capture_resid && upto < 0) caps["x" + std::to_string(i)] = x;
      if (!global) local_x = x;
      for (int o = 0; o < NL; ++o)
        if (c.out_layers[o] == i) {
          const int Cf = c.cat_token ? 2 * E : E;
          std::vector<float> f(static_cast<size_t>(S) * Np * Cf);
          const float* nw = F("vit.norm.weight");
          const float* nb = F("vit.norm.bias");
#pragma omp parallel for schedule(static)
          for (int row = 0; row < S * Np; ++row) {
            const int s = row / Np, tk = 1 + row % Np;
            const float* xr = &x[(static_cast<size_t>(s) * Nt + tk) * E];
            float* dst = &f[static_cast<size_t>(row) * Cf];
            if (c.cat_token) {
              const float* lr = &local_x[(static_cast<size_t>(s) * Nt + tk) * E];
              for (int e = 0; e < E; ++e) dst[e] = lr[e];
              layernorm_rows(xr, 1, E, nw, nb, c.ln_eps, dst + E);  // in-graph ggml_norm (:301)
            } else {
              layernorm_host(xr, E, nw, nb, c.ln_eps, dst);  // host double LN (:174-181)
            }
          }
          feats[o] = std::move(f);
          if (cams) {
            // camera token (src/dino_backbone.cpp:187-201, :598-601): token 0, raw (no norm):
            // cat(local_x, x) for cat-token models, x alone otherwise; [S][Cf]
            std::vector<float> cv(static_cast<size_t>(S) * Cf);
            for (int s2 = 0; s2 < S; ++s2) {
              const float* xr = &x[static_cast<size_t>(s2) * Nt * E];
              float* dst = &cv[static_cast<size_t>(s2) * Cf];
              if (c.cat_token) {
                const float* lr = &local_x[static_cast<size_t>(s2) * Nt * E];
                for (int e = 0; e < E; ++e) dst[e] = lr[e];
                for (int e = 0; e < E; ++e) dst[E + e] = xr[e];
              } else {
                for (int e = 0; e < E; ++e) dst[e] = xr[e];
              }
            }
            (*cams)[o] = std::move(cv);
          }
        }
    }
    if (x_out) *x_out = x;
  }

  // CamPose::pose (src/cam_pose.cpp:8-83): camera-token MLP -> pose encoding
  // [t(3), quaternion xyzw (4), fov h/w (2)] -> extrinsics (3x4 world-to-camera) and
  // intrinsics (3x3) at the processed size H x W. out[0..9) pose_enc, [9..21) ext,
  // [21..30) intr. Returns false without camera weights or on a width mismatch.
  bool pose(const float* cam_token, int D, int H, int W, float* out) {
    if (!has("cam.bb0.weight") || T("cam.bb0.weight").ne[0] != D) return false;
    auto lin = [&](const std::vector<float>& in, const std::string& n, bool relu) {
      const Tensor& w = T("cam." + n + ".weight");
      std::vector<float> y(static_cast<size_t>(w.ne[1]));
      linear(in.data(), 1, static_cast<int>(w.ne[0]), "cam." + n + ".weight", "cam." + n + ".bias", y.data());
      if (relu)
        for (auto& v : y) v = std::max(0.0f, v);
      return y;
    };
    std::vector<float> f(cam_token, cam_token + D);
    f = lin(f, "bb0", true);
    f = lin(f, "bb2", true);
    const std::vector<float> t3 = lin(f, "fc_t", false), q4 = lin(f, "fc_q", false), fv = lin(f, "fc_fov", true);
    const float pe[9] = {t3[0], t3[1], t3[2], q4[0], q4[1], q4[2], q4[3], fv[0], fv[1]};
    for (int i = 0; i < 9; ++i) out[i] = pe[i];
    const float qi = pe[3], qj = pe[4], qk = pe[5], qr = pe[6];
    const float sc = 2.0f / (qi * qi + qj * qj + qk * qk + qr * qr);
    const float R[3][3] = {{1.0f - sc * (qj * qj + qk * qk), sc * (qi * qj - qk * qr), sc * (qi * qk + qj * qr)},
                           {sc * (qi * qj + qk * qr), 1.0f - sc * (qi * qi + qk * qk), sc * (qj * qk - qi * qr)},
                           {sc * (qi * qk - qj * qr), sc * (qj * qk + qi * qr), 1.0f - sc * (qi * qi + qj * qj)}};
    const float fy = (H / 2.0f) / std::max(std::tan(pe[7] / 2.0f), 1e-6f);
    const float fx = (W / 2.0f) / std::max(std::tan(pe[8] / 2.0f), 1e-6f);
    float* ext = out + 9;
    float* intr = out + 21;
    for (int r = 0; r < 3; ++r) {
      float acc = 0.0f;
      for (int k = 0; k < 3; ++k) acc += R[k][r] * pe[k];
      for (int k = 0; k < 3; ++k) ext[r * 4 + k] = R[k][r];
      ext[r * 4 + 3] = -acc;
    }
    for (int i = 0; i < 9; ++i) intr[i] = 0.0f;
    intr[0] = fx;
    intr[4] = fy;
    intr[2] = W / 2.0f;
    intr[5] = H / 2.0f;
    intr[8] = 1.0f;
    return true;
  }

  // select_reference_view_saddle (src/dino_backbone.cpp:372-412).
  static int select_saddle(const std::vector<std::vector<float>>& cls, int E) {
    const int S = static_cast<int>(cls.size());
    if (S <= 1) return 0;
    std::vector<double> nrm(S), sim(S), fn(S), fv(S);
    std::vector<std::vector<double>> cn(S, std::vector<double>(E));
    for (int v = 0; v < S; ++v) {
      double n = 0;
      for (int e = 0; e < E; ++e) n += static_cast<double>(cls[v][e]) * cls[v][e];
      n = std::sqrt(n);
      nrm[v] = n;
      const double inv = n > 0 ? 1.0 / n : 0.0;
      for (int e = 0; e < E; ++e) cn[v][e] = cls[v][e] * inv;
    }
    for (int v = 0; v < S; ++v) {
      double s = 0;
      for (int w = 0; w < S; ++w) {
        if (w == v) continue;
        double dot = 0;
        for (int e = 0; e < E; ++e) dot += cn[v][e] * cn[w][e];
        s += dot;
      }
      sim[v] = s / (S - 1);
      fn[v] = nrm[v];
      double mean = 0;
      for (int e = 0; e < E; ++e) mean += cn[v][e];
      mean /= E;
      double var = 0;
      for (int e = 0; e < E; ++e) var += (cn[v][e] - mean) * (cn[v][e] - mean);
      fv[v] = var / (E - 1);
    }
    auto norm01 = [](std::vector<double>& m) {
      double mn = m[0], mx = m[0];
      for (double v : m) { mn = std::min(mn, v); mx = std::max(mx, v); }
      for (double& v : m) v = (v - mn) / (mx - mn + 1e-8);
    };
    norm01(sim);
    norm01(fn);
    norm01(fv);
    int best = 0;
    double bb = 1e300;
    for (int v = 0; v < S; ++v) {
      const double bal = std::fabs(sim[v] - 0.5) + std::fabs(fn[v] - 0.5) + std::fabs(fv[v] - 0.5);
      if (bal < bb) { bb = bal; best = v; }
    }
    return best;
  }
};

// ------------------------------------------------------------------ preprocessing
// (src/preprocess.cpp:8-197)
struct Img {
  int w = 0, h = 0;
  std::vector<uint8_t> rgb;
};
uint8_t sat_u8(float v) {
  long r = lrintf(v);
  return static_cast<uint8_t>(r < 0 ? 0 : (r > 255 ? 255 : r));
}
float cubic_w(float x) {
  const float a = -0.75f;
  x = std::fabs(x);
  if (x < 1) return ((a + 2) * x - (a + 3)) * x * x + 1;
  if (x < 2) return (((x - 5) * x + 8) * x - 4) * a;
  return 0.f;
}
void resize_bilinear(const Img& s, int dw, int dh, std::vector<float>& dst) {
  dst.assign(static_cast<size_t>(dw) * dh * 3, 0.f);
  const float sx = static_cast<float>(s.w) / dw, sy = static_cast<float>(s.h) / dh;
  for (int y = 0; y < dh; ++y) {
    const float fy = (y + 0.5f) * sy - 0.5f;
    const int y0 = static_cast<int>(std::floor(fy));
    const float wy = fy - y0;
    const int y0c = std::clamp(y0, 0, s.h - 1), y1c = std::clamp(y0 + 1, 0, s.h - 1);
    for (int x = 0; x < dw; ++x) {
      const float fx = (x + 0.5f) * sx - 0.5f;
      const int x0 = static_cast<int>(std::floor(fx));
      const float wx = fx - x0;
      const int x0c = std::clamp(x0, 0, s.w - 1), x1c = std::clamp(x0 + 1, 0, s.w - 1);
      for (int ch = 0; ch < 3; ++ch) {
        auto P = [&](int yy, int xx) { return static_cast<float>(s.rgb[(static_cast<size_t>(yy) * s.w + xx) * 3 + ch]); };
        const float top = P(y0c, x0c) * (1 - wx) + P(y0c, x1c) * wx;
        const float bot = P(y1c, x0c) * (1 - wx) + P(y1c, x1c) * wx;
        dst[(static_cast<size_t>(y) * dw + x) * 3 + ch] = top * (1 - wy) + bot * wy;
      }
    }
  }
}
Img resize_cubic(const Img& src, int dw, int dh) {
  Img dst;
  dst.w = dw;
  dst.h = dh;
  dst.rgb.assign(static_cast<size_t>(dw) * dh * 3, 0);
  const int sw = src.w, sh = src.h;
  const double sx = static_cast<double>(sw) / dw, sy = static_cast<double>(sh) / dh;
  std::vector<int> xi(static_cast<size_t>(dw) * 4);
  std::vector<float> xw(static_cast<size_t>(dw) * 4);
  for (int x = 0; x < dw; ++x) {
    const double fx = (x + 0.5) * sx - 0.5;
    const int ix = static_cast<int>(std::floor(fx));
    const float t = static_cast<float>(fx - ix);
    const float w[4] = {cubic_w(t + 1), cubic_w(t), cubic_w(t - 1), cubic_w(t - 2)};
    for (int k = 0; k < 4; ++k) {
      xi[x * 4 + k] = std::clamp(ix - 1 + k, 0, sw - 1);
      xw[x * 4 + k] = w[k];
    }
  }
  std::vector<float> tmp(static_cast<size_t>(sh) * dw * 3);
  for (int y = 0; y < sh; ++y)
    for (int x = 0; x < dw; ++x)
      for (int ch = 0; ch < 3; ++ch) {
        float acc = 0;
        for (int k = 0; k < 4; ++k) acc += xw[x * 4 + k] * static_cast<float>(src.rgb[(static_cast<size_t>(y) * sw + xi[x * 4 + k]) * 3 + ch]);
        tmp[(static_cast<size_t>(y) * dw + x) * 3 + ch] = acc;
      }
  for (int y = 0; y < dh; ++y) {
    const double fy = (y + 0.5) * sy - 0.5;
    const int iy = static_cast<int>(std::floor(fy));
    const float t = static_cast<float>(fy - iy);
    const float w[4] = {cubic_w(t + 1), cubic_w(t), cubic_w(t - 1), cubic_w(t - 2)};
    int yi[4];
    for (int k = 0; k < 4; ++k) yi[k] = std::clamp(iy - 1 + k, 0, sh - 1);
    for (int x = 0; x < dw; ++x)
      for (int ch = 0; ch < 3; ++ch) {
        float acc = 0;
        for (int k = 0; k < 4; ++k) acc += w[k] * tmp[(static_cast<size_t>(yi[k]) * dw + x) * 3 + ch];
        dst.rgb[(static_cast<size_t>(y) * dw + x) * 3 + ch] = sat_u8(acc);
      }
  }
  return dst;
}
struct AreaTap {
  int di, si;
  float alpha;
};
std::vector<AreaTap> area_tab(int ssize, int dsize) {
  std::vector<AreaTap> tab;
  const double scale = static_cast<double>(ssize) / dsize;
  for (int dx = 0; dx < dsize; ++dx) {
    const double fsx1 = dx * scale, fsx2 = fsx1 + scale;
    const double cw = std::min(scale, static_cast<double>(ssize) - fsx1);
    int sx1 = static_cast<int>(std::ceil(fsx1)), sx2 = static_cast<int>(std::floor(fsx2));
    sx2 = std::min(sx2, ssize - 1);
    sx1 = std::min(sx1, sx2);
    if (sx1 - fsx1 > 1e-3) tab.push_back({dx, sx1 - 1, static_cast<float>((sx1 - fsx1) / cw)});
    for (int sx = sx1; sx < sx2; ++sx) tab.push_back({dx, sx, static_cast<float>(1.0 / cw)});
    if (fsx2 - sx2 > 1e-3) tab.push_back({dx, sx2, static_cast<float>(std::min(std::min(fsx2 - sx2, 1.0), cw) / cw)});
  }
  return tab;
}
Img resize_area(const Img& src, int dw, int dh) {
  const int sw = src.w, sh = src.h;
  if (dw >= sw && dh >= sh) {
    Img up;
    std::vector<float> hwc;
    resize_bilinear(src, dw, dh, hwc);
    up.w = dw;
    up.h = dh;
    up.rgb.resize(hwc.size());
    for (size_t i = 0; i < hwc.size(); ++i) up.rgb[i] = sat_u8(hwc[i]);
    return up;
  }
  auto xt = area_tab(sw, dw), yt = area_tab(sh, dh);
  std::vector<float> tmp(static_cast<size_t>(sh) * dw * 3, 0.f);
  for (int y = 0; y < sh; ++y)
    for (const auto& t : xt)
      for (int ch = 0; ch < 3; ++ch)
        tmp[(static_cast<size_t>(y) * dw + t.di) * 3 + ch] += t.alpha * static_cast<float>(src.rgb[(static_cast<size_t>(y) * sw + t.si) * 3 + ch]);
  std::vector<float> acc(static_cast<size_t>(dh) * dw * 3, 0.f);
  for (const auto& t : yt)
    for (int x = 0; x < dw; ++x)
      for (int ch = 0; ch < 3; ++ch)
        acc[(static_cast<size_t>(t.di) * dw + x) * 3 + ch] += t.alpha * tmp[(static_cast<size_t>(t.si) * dw + x) * 3 + ch];
  Img dst;
  dst.w = dw;
  dst.h = dh;
  dst.rgb.resize(acc.size());
  for (size_t i = 0; i < acc.size(); ++i) dst.rgb[i] = sat_u8(acc[i]);
  return dst;
}
int nearest_multiple(int x, int p) {
  const int down = (x / p) * p, up = down + p;
  return (std::abs(up - x) <= std::abs(x - down)) ? up : down;
}
// preprocess_real / legacy preprocess -> CHW f32 normalised.
bool preprocess(const Img& img, const or_config& c, bool legacy, std::vector<float>& chw, int& H, int& W) {
  if (img.w <= 0 || img.h <= 0) return false;
  const int patch = c.patch_size;
  if (legacy) {
    int dw = (img.w / patch) * patch, dh = (img.h / patch) * patch;
    if (dw == 0) dw = patch;
    if (dh == 0) dh = patch;
    std::vector<float> hwc;
    resize_bilinear(img, dw, dh, hwc);
    W = dw;
    H = dh;
    chw.assign(static_cast<size_t>(3) * dh * dw, 0.f);
    for (int ch = 0; ch < 3; ++ch)
      for (int y = 0; y < dh; ++y)
        for (int x = 0; x < dw; ++x) {
          const float v = hwc[(static_cast<size_t>(y) * dw + x) * 3 + ch] / 255.f;
          chw[(static_cast<size_t>(ch) * dh + y) * dw + x] = (v - c.img_mean[ch]) / c.img_std[ch];
        }
    return true;
  }
  const int target = c.resize_target > 0 ? c.resize_target : 504;
  Img cur = img;
  {
    const int bound = c.resize_upper ? std::max(cur.w, cur.h) : std::min(cur.w, cur.h);
    if (bound != target) {
      const double scale = static_cast<double>(target) / bound;
      const int nw = std::max(1, static_cast<int>(std::nearbyint(cur.w * scale)));
      const int nh = std::max(1, static_cast<int>(std::nearbyint(cur.h * scale)));
      cur = scale > 1.0 ? resize_cubic(cur, nw, nh) : resize_area(cur, nw, nh);
    }
  }
  {
    const int nw = std::max(1, nearest_multiple(cur.w, patch)), nh = std::max(1, nearest_multiple(cur.h, patch));
    if (nw != cur.w || nh != cur.h) {
      const bool upscale = nw > cur.w || nh > cur.h;
      cur = upscale ? resize_cubic(cur, nw, nh) : resize_area(cur, nw, nh);
    }
  }
  H = cur.h;
  W = cur.w;
  chw.assign(static_cast<size_t>(3) * H * W, 0.f);
  for (int ch = 0; ch < 3; ++ch)
    for (int y = 0; y < H; ++y)
      for (int x = 0; x < W; ++x) {
        const float v = static_cast<float>(cur.rgb[(static_cast<size_t>(y) * W + x) * 3 + ch]) / 255.f;
        chw[(static_cast<size_t>(ch) * H + y) * W + x] = (v - c.img_mean[ch]) / c.img_std[ch];
      }
  return true;
}

struct Handle {
  Oracle o;
  std::vector<float> depth, conf, logits, aux, chw, pose, sky;
  std::vector<std::vector<float>> feats;
  int H = 0, W = 0, od = 0, aux_h = 0, aux_w = 0, b_idx = 0;
};

}  // namespace

// ====================================================================== C ABI
OR_API void* or_create(const or_config* cfg, const or_tensor* ts, int n) {
  auto* h = new Handle();
  h->o.c = *cfg;
  for (int i = 0; i < n; ++i) {
    Tensor t;
    t.data = ts[i].data;
    t.type = ts[i].type;
    for (int k = 0; k < 4; ++k) t.ne[k] = ts[i].ne[k] > 0 ? ts[i].ne[k] : 1;
    h->o.t[ts[i].name] = t;
  }
#ifdef _OPENMP
  if (cfg->n_threads > 0) omp_set_num_threads(cfg->n_threads);
#endif
  return h;
}

OR_API void or_destroy(void* p) { delete static_cast<Handle*>(p); }

// Model-free entry points for the DA3 host-code pins: the RoPE tables for explicit
// positions (src/rope2d.cpp:4-27), the offset bicubic pos-embed interpolation of an
// explicit table [1 + grid^2][embed] (src/dino_backbone.cpp:18-56), and the saddle
// reference-view choice from S CLS vectors [S][embed] (src/dino_backbone.cpp:372-412).
OR_API int or_rope_tables(const float* pos_yx, int tokens, int head_dim, float freq, float* cos_out, float* sin_out) {
  Oracle o;
  o.c.head_dim = head_dim;
  o.c.rope_freq = freq;
  const std::vector<float> pos(pos_yx, pos_yx + static_cast<size_t>(tokens) * 2);
  const Oracle::Rope r = o.rope_tables(pos, tokens);
  memcpy(cos_out, r.cos.data(), r.cos.size() * sizeof(float));
  memcpy(sin_out, r.sin.data(), r.sin.size() * sizeof(float));
  return 0;
}

OR_API int or_interp_pos_embed(const float* pos_embed, int embed, int grid, float offset, int gh, int gw, float* out) {
  Oracle o;
  o.c.embed_dim = embed;
  o.c.pos_embed_grid = grid;
  o.c.interp_offset = offset;
  Tensor t;
  t.data = pos_embed;
  t.type = 0;
  t.ne[0] = embed;
  t.ne[1] = 1 + grid * grid;
  o.t["vit.pos_embed"] = t;
  const std::vector<float> v = o.interp_pos_embed(gh, gw);
  memcpy(out, v.data(), v.size() * sizeof(float));
  return 0;
}

// linear() (src/ggml_extend.hpp:6-10) of x f32 [M][K] with a Q8_0 weight given as GGUF
// bytes [N][K/32][34] and an optional f32 bias [N]: act_quant = 1 follows ggml's Q8_0 x
// Q8_0 CPU dot product, 0 the f32 path. y f32 [M][N].
OR_API int or_linear_q8(const float* x, int M, int K, const uint8_t* wq8, int N, const float* bias, int act_quant,
                        float* y) {
  Oracle o;
  o.c.act_quant = act_quant;
  Tensor w;
  w.data = wq8;
  w.type = 8;
  w.ne[0] = K;
  w.ne[1] = N;
  o.t["w"] = w;
  if (bias) {
    Tensor b;
    b.data = bias;
    b.type = 0;
    b.ne[0] = N;
    o.t["b"] = b;
  }
  o.linear(x, M, K, "w", bias ? "b" : "", y);
  return 0;
}

OR_API int or_select_saddle(const float* cls, int S, int embed) {
  std::vector<std::vector<float>> c(S);
  for (int s = 0; s < S; ++s) c[s].assign(cls + static_cast<size_t>(s) * embed, cls + static_cast<size_t>(s + 1) * embed);
  return Oracle::select_saddle(c, embed);
}

// 1: later forwards keep the residual stream after every block (or_get "x<i>",
// [S * tokens][embed] in processing order); 0: off.
OR_API void or_set_capture_resid(void* p, int on) { static_cast<Handle*>(p)->o.capture_resid = on != 0; }

OR_API void or_quantize_q8_0(const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 32; ++b) {
    float d;
    int8_t q[32];
    quantize_row(x + b * 32, 32, &d, q);
    // re-derive the exact stored fp16 scale (quantize_row returns it widened)
    const uint16_t dh = f2h(d);
    memcpy(out + b * 34, &dh, 2);
    memcpy(out + b * 34 + 2, q, 32);
  }
}

OR_API int or_preprocess(void* p, const uint8_t* rgb, int w, int hgt, int legacy, float* out, int* H, int* W) {
  auto* h = static_cast<Handle*>(p);
  Img img;
  img.w = w;
  img.h = hgt;
  img.rgb.assign(rgb, rgb + static_cast<size_t>(w) * hgt * 3);
  std::vector<float> chw;
  if (!preprocess(img, h->o.c, legacy != 0, chw, *H, *W)) return -1;
  if (out) memcpy(out, chw.data(), chw.size() * 4);
  return 0;
}

// Model-free entry points for the preprocessing pins: the same preprocess with the
// policy given explicitly, the two uint8 resizers (mode 0 cubic, 1 area), and the raw
// UV embedding in the reference's [ph][pw][C] order (src/uv_posembed.hpp:4-7).
OR_API int or_preprocess_cfg(const uint8_t* rgb, int w, int hgt, int patch, int target, int upper, const float* mean,
                             const float* std_, int legacy, float* out, int64_t cap, int* H, int* W) {
  or_config c{};
  c.patch_size = patch;
  c.resize_target = target;
  c.resize_upper = upper;
  for (int i = 0; i < 3; ++i) {
    c.img_mean[i] = mean[i];
    c.img_std[i] = std_[i];
  }
  Img img;
  img.w = w;
  img.h = hgt;
  img.rgb.assign(rgb, rgb + static_cast<size_t>(w) * hgt * 3);
  std::vector<float> chw;
  if (!preprocess(img, c, legacy != 0, chw, *H, *W)) return -1;
  if (static_cast<int64_t>(chw.size()) > cap) return -2;
  memcpy(out, chw.data(), chw.size() * 4);
  return 0;
}

OR_API int or_resize(const uint8_t* rgb, int w, int hgt, int dw, int dh, int mode, uint8_t* out) {
  Img img;
  img.w = w;
  img.h = hgt;
  img.rgb.assign(rgb, rgb + static_cast<size_t>(w) * hgt * 3);
  const Img r = mode == 0 ? resize_cubic(img, dw, dh) : resize_area(img, dw, dh);
  memcpy(out, r.rgb.data(), r.rgb.size());
  return 0;
}

OR_API int or_uv_pos_embed(int pw, int ph, int C, float aspect, float* out) {
  const Oracle::Map m = Oracle::uv_embed(pw, ph, C, aspect, 1.0f);
  const size_t hw = static_cast<size_t>(pw) * ph;
  for (int ch = 0; ch < C; ++ch)
    for (size_t p = 0; p < hw; ++p) out[p * C + ch] = m.v[ch * hw + p];
  return 0;
}

// Single image: RGB8 HWC -> depth (+conf) at the processed size.
// DA2 route: preprocess_real -> forward -> depth_relative (src/engine.cpp:121-130,
// src/dpt_head.cpp:402-439); DA3 route: preprocess_real -> fused feats -> head ->
// exp / exp+1 (src/engine.cpp:189-229). legacy=1 uses the floor-to-patch preprocess.
namespace {
// Forward + head + output activations of one normalised planar image held in h->chw
// (src/engine.cpp:189-229; mono: src/engine.cpp:105-115 and the sky relu of
// src/dpt_head.cpp:334-338).
int infer_chw(Handle* h, int H, int W, int want_aux) {
  struct Dump {
    ~Dump() { prof_dump("infer"); }
  } dump_;
  Oracle& o = h->o;
  h->H = H;
  h->W = W;
  std::vector<std::vector<float>> views{h->chw};
  std::vector<std::vector<float>> cams;
  o.backbone(views, H, W, h->feats, -1, nullptr, &cams);
  if (static_cast<int>(h->feats.size()) < 4) return -2;
  const int Cf = (o.c.cat_token ? 2 : 1) * o.c.embed_dim;
  h->pose.assign(30, 0.f);
  if (!o.pose(cams[3].data(), Cf, H, W, h->pose.data())) h->pose.clear();
  std::vector<const float*> f4 = {h->feats[0].data(), h->feats[1].data(), h->feats[2].data(), h->feats[3].data()};
  Oracle::Map aux, sky;
  Oracle::Map lg = o.head(f4, Cf, H, W, want_aux != 0, &aux, "", &sky);
  h->od = lg.C;
  h->logits = lg.v;
  const size_t HW = static_cast<size_t>(H) * W;
  h->depth.assign(HW, 0.f);
  h->conf.clear();
  if (o.c.is_da2) {
    for (size_t i = 0; i < HW; ++i)
      h->depth[i] = o.c.head_max_depth > 0.f ? (1.0f / (1.0f + std::exp(-lg.v[i]))) * o.c.head_max_depth : std::max(0.0f, lg.v[i]);
  } else {
    for (size_t i = 0; i < HW; ++i) h->depth[i] = std::exp(lg.v[i]);
    if (lg.C >= 2) {
      h->conf.resize(HW);
      for (size_t i = 0; i < HW; ++i) h->conf[i] = std::exp(lg.v[HW + i]) + 1.0f;
    }
  }
  h->sky.clear();
  if (sky.v.size() == HW) {
    h->sky.resize(HW);
    for (size_t i = 0; i < HW; ++i) h->sky[i] = std::max(0.0f, sky.v[i]);
  }
  h->aux = aux.v;
  h->aux_h = aux.H;
  h->aux_w = aux.W;
  return 0;
}
}  // namespace

// Single image: RGB8 HWC -> depth (+conf, +sky) at the processed size.
// DA2 route: preprocess_real -> forward -> depth_relative (src/engine.cpp:121-130,
// src/dpt_head.cpp:402-439); DA3 route: preprocess_real -> fused feats -> head ->
// exp / exp+1 (src/engine.cpp:189-229). legacy=1 uses the floor-to-patch preprocess.
OR_API int or_infer(void* p, const uint8_t* rgb, int w, int hgt, int legacy, int want_aux) {
  auto* h = static_cast<Handle*>(p);
  Img img;
  img.w = w;
  img.h = hgt;
  img.rgb.assign(rgb, rgb + static_cast<size_t>(w) * hgt * 3);
  int H = 0, W = 0;
  if (!preprocess(img, h->o.c, legacy != 0, h->chw, H, W)) return -1;
  return infer_chw(h, H, W, want_aux);
}

// The same from an already normalised planar f32 image [3][H][W] (the input the nested
// path shares between its two branches, src/engine.cpp:418-421).
OR_API int or_infer_chw(void* p, const float* chw, int H, int W, int want_aux) {
  auto* h = static_cast<Handle*>(p);
  const int P = h->o.c.patch_size;
  if (H <= 0 || W <= 0 || H % P || W % P) return -1;
  h->chw.assign(chw, chw + static_cast<size_t>(3) * H * W);
  return infer_chw(h, H, W, want_aux);
}

// Multi-view (S views, same size): src/engine.cpp:352-384 + forward_mv
// (src/dino_backbone.cpp:414-460) with the per-view depth head (+ aux rays).
// Outputs are concatenated per view in the original order.
OR_API int or_infer_mv(void* p, const uint8_t* const* rgbs, int S, int w, int hgt, int legacy, int want_aux) {
  auto* h = static_cast<Handle*>(p);
  Oracle& o = h->o;
  std::vector<std::vector<float>> views(S);
  int H = 0, W = 0;
  for (int s = 0; s < S; ++s) {
    Img img;
    img.w = w;
    img.h = hgt;
    img.rgb.assign(rgbs[s], rgbs[s] + static_cast<size_t>(w) * hgt * 3);
    int h2 = 0, w2 = 0;
    if (!preprocess(img, o.c, legacy != 0, views[s], h2, w2)) return -1;
    if (s == 0) { H = h2; W = w2; }
    else if (h2 != H || w2 != W) return -2;
  }
  h->H = H;
  h->W = W;
  const int E = o.c.embed_dim, P = o.c.patch_size, Nt = 1 + (H / P) * (W / P);
  int b_idx = 0;
  std::vector<int> order(S);
  for (int s = 0; s < S; ++s) order[s] = s;
  if (S >= 3 && o.c.alt_start >= 0) {
    std::vector<float> xa;
    std::vector<std::vector<float>> dummy;
    o.backbone(views, H, W, dummy, o.c.alt_start - 1, &xa);
    std::vector<std::vector<float>> cls(S, std::vector<float>(E));
    for (int s = 0; s < S; ++s)
      for (int e = 0; e < E; ++e) cls[s][e] = xa[static_cast<size_t>(s) * Nt * E + e];
    b_idx = Oracle::select_saddle(cls, E);
    order[0] = b_idx;
    for (int q = 1; q < S; ++q) order[q] = q <= b_idx ? q - 1 : q;
  }
  h->b_idx = b_idx;
  std::vector<std::vector<float>> rv(S);
  for (int q = 0; q < S; ++q) rv[q] = views[order[q]];
  std::vector<std::vector<float>> feats, cams;
  o.backbone(rv, H, W, feats, -1, nullptr, &cams);
  const int Cf = (o.c.cat_token ? 2 : 1) * E;
  const int Np = Nt - 1;
  h->pose.assign(static_cast<size_t>(S) * 30, 0.f);
  const size_t HW = static_cast<size_t>(H) * W;
  h->depth.assign(HW * S, 0.f);
  h->conf.assign(HW * S, 0.f);
  h->logits.clear();
  h->aux.clear();
  h->feats.assign(4, std::vector<float>(static_cast<size_t>(S) * Np * Cf));
  for (int t = 0; t < S; ++t) {
    // original view t sits at processing position q with order[q] == t
    int q = 0;
    while (order[q] != t) ++q;
    std::vector<const float*> f4;
    for (int l = 0; l < 4; ++l) {
      f4.push_back(&feats[l][static_cast<size_t>(q) * Np * Cf]);
      memcpy(&h->feats[l][static_cast<size_t>(t) * Np * Cf], f4.back(), static_cast<size_t>(Np) * Cf * 4);
    }
    if (!o.pose(&cams[3][static_cast<size_t>(q) * Cf], Cf, H, W, &h->pose[static_cast<size_t>(t) * 30])) h->pose.clear();
    Oracle::Map aux;
    Oracle::Map lg = o.head(f4, Cf, H, W, want_aux != 0, &aux, "v" + std::to_string(t) + ".");
    h->od = lg.C;
    for (size_t i = 0; i < HW; ++i) {
      h->depth[t * HW + i] = std::exp(lg.v[i]);
      if (lg.C >= 2) h->conf[t * HW + i] = std::exp(lg.v[HW + i]) + 1.0f;
    }
    h->logits.insert(h->logits.end(), lg.v.begin(), lg.v.end());
    h->aux.insert(h->aux.end(), aux.v.begin(), aux.v.end());
    h->aux_h = aux.H;
    h->aux_w = aux.W;
  }
  return 0;
}

// Accessors: name in {"depth","conf","logits","aux","chw","pose","feat0".."feat3"} or a
// capture key ("stage0".."stage3","out1", "v<k>.stage0"...). Returns element count.
OR_API int64_t or_get(void* p, const char* name, const float** out) {
  auto* h = static_cast<Handle*>(p);
  std::string n(name);
  const std::vector<float>* v = nullptr;
  if (n == "depth") v = &h->depth;
  else if (n == "conf") v = &h->conf;
  else if (n == "logits") v = &h->logits;
  else if (n == "aux") v = &h->aux;
  else if (n == "chw") v = &h->chw;
  else if (n == "pose") v = &h->pose;
  else if (n == "sky") v = &h->sky;
  else if (n.size() == 5 && n.compare(0, 4, "feat") == 0) {
    const int l = n[4] - '0';
    if (l >= 0 && l < static_cast<int>(h->feats.size())) v = &h->feats[l];
  } else {
    auto it = h->o.caps.find(n);
    if (it != h->o.caps.end()) v = &it->second;
  }
  if (!v) { *out = nullptr; return -1; }
  *out = v->data();
  return static_cast<int64_t>(v->size());
}

OR_API void or_dims(void* p, int* H, int* W, int* od, int* aux_h, int* aux_w, int* b_idx) {
  auto* h = static_cast<Handle*>(p);
  *H = h->H;
  *W = h->W;
  *od = h->od;
  *aux_h = h->aux_h;
  *aux_w = h->aux_w;
  *b_idx = h->b_idx;
}

// ====================================================================== nested metric alignment
// Restatement of NestedAligner (src/nested.cpp:7-96) for the checker: torch.quantile with
// linear interpolation over a full sort, the mono sky fill, then the alignment.
namespace {
float or_quantile(std::vector<float> v, float q) {  // src/nested.cpp:7-20
  if (v.empty()) return 0.0f;
  std::sort(v.begin(), v.end());
  const size_t n = v.size();
  if (n == 1) return v[0];
  const double pos = static_cast<double>(q) * static_cast<double>(n - 1);
  const double fl = std::floor(pos);
  const size_t i0 = static_cast<size_t>(fl);
  const size_t i1 = std::min(static_cast<size_t>(std::ceil(pos)), n - 1);
  return static_cast<float>(static_cast<double>(v[i0]) + (pos - fl) * (static_cast<double>(v[i1]) - static_cast<double>(v[i0])));
}
}  // namespace

// metric_depth is sky-filled in place (src/nested.cpp:22-33) before the alignment
// (src/nested.cpp:35-96); returns the scale factor.
OR_API float or_nested_align(const float* any_depth, const float* any_conf, const float* any_ext, const float* any_intr,
                             float* metric_depth, const float* sky, int64_t n, float* out_depth, float* out_ext) {
  const size_t N = static_cast<size_t>(n);
  {
    std::vector<float> ns;
    size_t n_sky = 0;
    for (size_t i = 0; i < N; ++i) {
      if (sky[i] < 0.3f) ns.push_back(metric_depth[i]);
      else ++n_sky;
    }
    if (ns.size() > 10 && n_sky > 10) {
      const float v = or_quantile(ns, 0.99f);
      for (size_t i = 0; i < N; ++i)
        if (!(sky[i] < 0.3f)) metric_depth[i] = v;
    }
  }
  const float focal = (any_intr[0] + any_intr[4]) * 0.5f;
  const float mscale = focal / 300.0f;
  std::vector<float> conf_ns;
  for (size_t i = 0; i < N; ++i)
    if (sky[i] < 0.3f) conf_ns.push_back(any_conf[i]);
  const float med = or_quantile(conf_ns, 0.5f);
  double num = 0.0, den = 0.0;
  for (size_t i = 0; i < N; ++i) {
    const float md = metric_depth[i] * mscale;
    if (sky[i] < 0.3f && any_conf[i] >= med && md > 1e-2f && any_depth[i] > 1e-3f) {
      num += static_cast<double>(md) * static_cast<double>(any_depth[i]);
      den += static_cast<double>(any_depth[i]) * static_cast<double>(any_depth[i]);
    }
  }
  if (den < 1e-12) den = 1e-12;
  const float sf = static_cast<float>(num / den);
  for (int k = 0; k < 12; ++k) out_ext[k] = any_ext[k];
  out_ext[3] *= sf;
  out_ext[7] *= sf;
  out_ext[11] *= sf;
  std::vector<float> d_ns;
  for (size_t i = 0; i < N; ++i) {
    out_depth[i] = any_depth[i] * sf;
    if (sky[i] < 0.3f) d_ns.push_back(out_depth[i]);
  }
  float cap = or_quantile(d_ns, 0.99f);
  if (cap > 200.0f) cap = 200.0f;
  for (size_t i = 0; i < N; ++i)
    if (!(sky[i] < 0.3f)) out_depth[i] = cap;
  return sf;
}

// ====================================================================== ray -> pose solver
// Restatement of the host ray->pose solver (src/ray_pose.cpp:11-252, src/linalg.cpp:8-203)
// for the checker: dense double linear algebra on 3x3 / 9x9 matrices, a weighted
// homography RANSAC over the aux ray field, QL of the refit homography. Operation order
// follows the reference so the double results agree to the bit.
namespace {
namespace rp {

double sgn(double x) { return static_cast<double>((x > 0.0) - (x < 0.0)); }

double det3(const double* a) {  // src/linalg.cpp:10-14
  return a[0] * (a[4] * a[8] - a[5] * a[7]) - a[1] * (a[3] * a[8] - a[5] * a[6]) + a[2] * (a[3] * a[7] - a[4] * a[6]);
}

// Householder QR of an n x n row-major matrix with n-1 reflectors (LAPACK sign
// convention, last diagonal untouched) (src/linalg.cpp:45-90).
void qr(const double* a, int n, double* q, double* r) {
  std::copy(a, a + n * n, r);
  for (int i = 0; i < n * n; ++i) q[i] = (i / n == i % n) ? 1.0 : 0.0;
  std::vector<double> v(n);
  for (int k = 0; k + 1 < n; ++k) {
    double nx = 0;
    for (int i = k; i < n; ++i) nx += r[i * n + k] * r[i * n + k];
    nx = std::sqrt(nx);
    if (nx < 1e-300) continue;
    const double alpha = r[k * n + k] >= 0.0 ? -nx : nx;
    std::fill(v.begin(), v.end(), 0.0);
    for (int i = k; i < n; ++i) v[i] = r[i * n + k];
    v[k] -= alpha;
    double vv = 0;
    for (int i = k; i < n; ++i) vv += v[i] * v[i];
    if (vv < 1e-300) continue;
    for (int j = 0; j < n; ++j) {  // R <- (I - 2vv'/vv) R
      double d = 0;
      for (int i = k; i < n; ++i) d += v[i] * r[i * n + j];
      const double f = 2.0 * d / vv;
      for (int i = k; i < n; ++i) r[i * n + j] -= f * v[i];
    }
    for (int row = 0; row < n; ++row) {  // Q <- Q (I - 2vv'/vv)
      double d = 0;
      for (int i = k; i < n; ++i) d += q[row * n + i] * v[i];
      const double f = 2.0 * d / vv;
      for (int i = k; i < n; ++i) q[row * n + i] -= f * v[i];
    }
  }
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < i; ++j) r[i * n + j] = 0.0;
}

// QL through QR of the column-reversed matrix, sign-normalised so diag(L) >= 0
// (src/linalg.cpp:96-126).
void ql3(const double* a, double* q, double* l) {
  double ar[9], qr_q[9], qr_r[9];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) ar[i * 3 + j] = a[i * 3 + 2 - j];
  qr(ar, 3, qr_q, qr_r);
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      q[i * 3 + j] = qr_q[i * 3 + 2 - j];
      l[i * 3 + j] = qr_r[(2 - i) * 3 + 2 - j];
    }
  const double s[3] = {sgn(l[0]), sgn(l[4]), sgn(l[8])};
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      q[i * 3 + j] *= s[j];
      l[i * 3 + j] *= s[i];
    }
}

// Cyclic Jacobi eigen-decomposition of a symmetric n x n matrix, eigenvectors in the
// columns of vec (src/linalg.cpp:128-172).
void jacobi(const double* m, int n, double* val, double* vec) {
  std::vector<double> a(m, m + n * n);
  for (int i = 0; i < n * n; ++i) vec[i] = (i / n == i % n) ? 1.0 : 0.0;
  for (int sweep = 0; sweep < 100; ++sweep) {
    double off = 0;
    for (int p = 0; p < n; ++p)
      for (int q = p + 1; q < n; ++q) off += a[p * n + q] * a[p * n + q];
    if (off < 1e-30) break;
    for (int p = 0; p < n; ++p)
      for (int q = p + 1; q < n; ++q) {
        const double apq = a[p * n + q];
        if (std::fabs(apq) < 1e-300) continue;
        const double theta = (a[q * n + q] - a[p * n + p]) / (2.0 * apq);
        double t = sgn(theta) / (std::fabs(theta) + std::sqrt(theta * theta + 1.0));
        if (theta == 0.0) t = 1.0;
        const double c = 1.0 / std::sqrt(t * t + 1.0), s = t * c;
        for (int i = 0; i < n; ++i) {
          const double x = a[i * n + p], y = a[i * n + q];
          a[i * n + p] = c * x - s * y;
          a[i * n + q] = s * x + c * y;
        }
        for (int i = 0; i < n; ++i) {
          const double x = a[p * n + i], y = a[q * n + i];
          a[p * n + i] = c * x - s * y;
          a[q * n + i] = s * x + c * y;
        }
        for (int i = 0; i < n; ++i) {
          const double x = vec[i * n + p], y = vec[i * n + q];
          vec[i * n + p] = c * x - s * y;
          vec[i * n + q] = s * x + c * y;
        }
      }
  }
  for (int i = 0; i < n; ++i) val[i] = a[i * n + i];
}

void smallest_vec(const double* m, int n, double* v) {  // src/linalg.cpp:174-181
  std::vector<double> val(n), vec(n * n);
  jacobi(m, n, val.data(), vec.data());
  int k = 0;
  for (int i = 1; i < n; ++i)
    if (val[i] < val[k]) k = i;
  for (int i = 0; i < n; ++i) v[i] = vec[i * n + k];
}

// Weighted DLT homography: smallest eigenvector of A'A, normalised by H[2][2]
// (src/linalg.cpp:183-203).
bool homography(const double* src, const double* dst, const double* w, int M, double* H) {
  double ata[81] = {0};
  for (int m = 0; m < M; ++m) {
    const double x = src[2 * m], y = src[2 * m + 1], u = dst[2 * m], v = dst[2 * m + 1];
    const double sw = std::sqrt(w[m] < 0 ? 0.0 : w[m]);
    const double a[9] = {-x * sw, -y * sw, -sw, 0, 0, 0, x * u * sw, y * u * sw, u * sw};
    const double b[9] = {0, 0, 0, -x * sw, -y * sw, -sw, x * v * sw, y * v * sw, v * sw};
    for (int i = 0; i < 9; ++i)
      for (int j = 0; j < 9; ++j) ata[i * 9 + j] += a[i] * a[j] + b[i] * b[j];
  }
  double h[9];
  smallest_vec(ata, 9, h);
  if (std::fabs(h[8]) < 1e-300) return false;
  const double inv = 1.0 / h[8];
  for (int i = 0; i < 9; ++i) H[i] = h[i] * inv;
  return true;
}

}  // namespace rp
}  // namespace

OR_API void or_qr(const double* a, int n, double* q, double* r) { rp::qr(a, n, q, r); }
OR_API void or_ql3(const double* a, double* q, double* l) { rp::ql3(a, q, l); }
OR_API void or_smallest_eigvec(const double* m, int n, double* v) { rp::smallest_vec(m, n, v); }
OR_API int or_homography(const double* src, const double* dst, const double* w, int M, double* H) {
  return rp::homography(src, dst, w, M, H) ? 0 : -1;
}

// Full solver on an interleaved ray field ray [Hy][Wx][6] (direction xyz, origin xyz)
// and confidence [Hy][Wx] (src/ray_pose.cpp:95-252 with its production defaults: 100
// iterations of 8 samples from the top 30 % by weight, reprojection threshold 0.2,
// at most 8000 refit points, seed 1234). ext = camera-to-world 3x4, intr 3x3. diag
// (optional, 26 doubles) = R (9), T (3), focal (2), pp (2), A (9), best inlier count.
// Returns 0, or -1 on a degenerate field.
OR_API int or_ray_pose(const float* ray, const float* conf, int Hy, int Wx, int img_h, int img_w, float* ext,
                       float* intr, double* diag) {
  const int N = Hy * Wx, n_iter = 100, n_pick = 8, max_refit = 8000;
  const double thr = 0.2, zthr = 1e-4;
  const uint32_t seed = 1234;
  // ray cloud on the identity camera plane (src/ray_pose.cpp:11-59)
  std::vector<double> src(2 * N), dst(2 * N), w(N), org(3 * N), craw(N);
  const double dx = 1.0 / Wx, dy = 1.0 / Hy;
  for (int i = 0; i < Hy; ++i) {
    const double gy = Hy == 1 ? dy : dy + static_cast<double>(i) * ((2.0 - dy) - dy) / (Hy - 1);
    for (int j = 0; j < Wx; ++j) {
      const double gx = Wx == 1 ? dx : dx + static_cast<double>(j) * ((2.0 - dx) - dx) / (Wx - 1);
      const int n = i * Wx + j;
      const float* r = ray + static_cast<size_t>(n) * 6;
      const double dz = r[2];
      const bool ok = std::fabs(dz) > zthr;
      src[2 * n] = gx - 1.0;
      src[2 * n + 1] = gy - 1.0;
      dst[2 * n] = ok ? r[0] / dz : static_cast<double>(r[0]);
      dst[2 * n + 1] = ok ? r[1] / dz : static_cast<double>(r[1]);
      craw[n] = conf[n];
      w[n] = ok ? craw[n] : 0.0;
      for (int c = 0; c < 3; ++c) org[3 * n + c] = r[3 + c];
    }
  }
  const int n_cand = std::min(N, std::max(n_pick, static_cast<int>(static_cast<double>(N) * 0.3)));
  std::vector<int> order(N);
  for (int n = 0; n < N; ++n) order[n] = n;
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return w[a] > w[b]; });
  // sample draws: one persistent permutation, partially re-shuffled per iteration
  std::vector<int> draws(static_cast<size_t>(n_iter) * n_pick), perm(n_cand);
  {
    std::mt19937 gen(seed);
    for (int k = 0; k < n_cand; ++k) perm[k] = k;
    for (int it = 0; it < n_iter; ++it)
      for (int k = 0; k < n_pick; ++k) {
        std::uniform_int_distribution<int> pick(k, n_cand - 1);
        std::swap(perm[k], perm[pick(gen)]);
        draws[static_cast<size_t>(it) * n_pick + k] = perm[k];
      }
  }
  auto fit = [&](const int* idx, int M, double* H) {
    std::vector<double> s(2 * M), d(2 * M), ww(M);
    for (int k = 0; k < M; ++k) {
      const int n = idx[k];
      s[2 * k] = src[2 * n];
      s[2 * k + 1] = src[2 * n + 1];
      d[2 * k] = dst[2 * n];
      d[2 * k + 1] = dst[2 * n + 1];
      ww[k] = w[n];
    }
    return rp::homography(s.data(), d.data(), ww.data(), M, H);
  };
  std::vector<uint8_t> best(N, 0), cur(N, 0);
  double best_score = -1.0;
  std::vector<int> sample(n_pick);
  for (int it = 0; it < n_iter; ++it) {
    for (int k = 0; k < n_pick; ++k) sample[k] = order[draws[static_cast<size_t>(it) * n_pick + k]];
    double H[9];
    if (!fit(sample.data(), n_pick, H)) continue;
    double score = 0;
    for (int n = 0; n < N; ++n) {
      const double x = src[2 * n], y = src[2 * n + 1];
      const double pz = H[6] * x + H[7] * y + H[8];
      const double ex = (H[0] * x + H[1] * y + H[2]) / pz - dst[2 * n];
      const double ey = (H[3] * x + H[4] * y + H[5]) / pz - dst[2 * n + 1];
      cur[n] = (ex * ex + ey * ey) < thr * thr;
      if (cur[n]) score += w[n];
    }
    if (score > best_score) {
      best_score = score;
      best = cur;
    }
  }
  std::vector<int> inl;
  for (int n = 0; n < N; ++n)
    if (best[n]) inl.push_back(n);
  const int n_best = static_cast<int>(inl.size());
  std::stable_sort(inl.begin(), inl.end(), [&](int a, int b) { return w[a] > w[b]; });
  if (static_cast<int>(inl.size()) > max_refit) {
    const int keep = std::max(static_cast<int>(inl.size() * 0.95), max_refit);
    inl.resize(keep);
    std::mt19937 gen(seed ^ 0x9e3779b9u);
    std::shuffle(inl.begin(), inl.end(), gen);
    inl.resize(max_refit);
  }
  if (inl.size() < 4) return -1;
  double A[9];
  if (!fit(inl.data(), static_cast<int>(inl.size()), A)) return -1;
  if (rp::det3(A) < 0)
    for (double& a : A) a = -a;
  double R[9], L[9];
  rp::ql3(A, R, L);
  const double l22 = L[8];
  if (std::fabs(l22) < 1e-12) return -1;
  for (double& v : L) v /= l22;
  if (std::fabs(L[0]) < 1e-12 || std::fabs(L[4]) < 1e-12) return -1;
  double T[3] = {0, 0, 0}, cs = 0;
  for (int n = 0; n < N; ++n) {
    for (int c = 0; c < 3; ++c) T[c] += org[3 * n + c] * craw[n];
    cs += craw[n];
  }
  if (std::fabs(cs) < 1e-12) return -1;
  for (double& t : T) t /= cs;
  const double focal[2] = {1.0 / L[0], 1.0 / L[4]}, pp[2] = {L[6] + 1.0, L[7] + 1.0};
  for (int i = 0; i < 3; ++i) {
    double t = 0;
    for (int c = 0; c < 3; ++c) {
      ext[i * 4 + c] = static_cast<float>(R[c * 3 + i]);  // rotation transposed: world from camera
    }
    t = -(R[0 * 3 + i] * T[0] + R[1 * 3 + i] * T[1] + R[2 * 3 + i] * T[2]);
    ext[i * 4 + 3] = static_cast<float>(t);
  }
  for (int k = 0; k < 9; ++k) intr[k] = 0.0f;
  intr[0] = static_cast<float>(focal[0] / 2.0 * img_w);
  intr[4] = static_cast<float>(focal[1] / 2.0 * img_h);
  intr[2] = static_cast<float>(pp[0] * img_w * 0.5);
  intr[5] = static_cast<float>(pp[1] * img_h * 0.5);
  intr[8] = 1.0f;
  for (int k = 0; k < 12; ++k)
    if (!std::isfinite(ext[k])) return -1;
  for (int k = 0; k < 9; ++k)
    if (!std::isfinite(intr[k])) return -1;
  if (diag) {
    std::copy(R, R + 9, diag);
    std::copy(T, T + 3, diag + 9);
    diag[12] = focal[0];
    diag[13] = focal[1];
    diag[14] = pp[0];
    diag[15] = pp[1];
    std::copy(A, A + 9, diag + 16);
    diag[25] = n_best;
  }
  return 0;
}
