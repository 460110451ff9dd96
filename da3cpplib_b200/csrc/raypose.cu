// Ray -> pose solver (src/ray_pose.cpp:95-252, src/linalg.cpp:8-203) on the GPU.
// Built with -fmad=false: every double expression below rounds exactly like the
// reference's host code (x86-64 baseline, no contraction), so the GPU cloud, fits,
// masks and ordered sums equal the reference's values bit for bit.
#include <math.h>
#include <string.h>

#include <algorithm>
#include <numeric>
#include <random>

#include "raypose.h"

namespace da3b {
namespace {

constexpr int kIter = 100;            // RANSAC iterations (src/ray_pose.hpp:12)
constexpr int kPick = 8;              // points per hypothesis
constexpr double kRatio = 0.3;        // candidate pool = top 30 % by weight
constexpr double kThr = 0.2;          // reprojection threshold
constexpr int kMaxRefit = 8000;       // refit subsample cap
constexpr double kZThr = 1e-4;        // |direction z| validity threshold
constexpr uint32_t kSeed = 1234;      // deterministic sampling seed
constexpr int kTile = 4096;           // radix-sort items per block (16 rounds of 256)

// ------------------------------------------------------------ shared double helpers
__host__ __device__ inline double sgn(double x) { return static_cast<double>((x > 0.0) - (x < 0.0)); }

// Identity-plane coordinate of grid index k of n: linspace(1/n, 2 - 1/n, n)[k] - 1
// (src/ray_pose.cpp:23-31).
__host__ __device__ inline double plane(int k, int n) {
  const double d = 1.0 / n;
  const double g = n == 1 ? d : d + static_cast<double>(k) * ((2.0 - d) - d) / (n - 1);
  return g - 1.0;
}

// One point's two rows of the weighted DLT system (src/linalg.cpp:190-196).
__host__ __device__ inline void dlt_rows(double x, double y, double u, double v, double w, double* a, double* b) {
  const double sw = sqrt(w < 0 ? 0.0 : w);
  a[0] = -x * sw; a[1] = -y * sw; a[2] = -sw; a[3] = 0; a[4] = 0; a[5] = 0;
  a[6] = x * u * sw; a[7] = y * u * sw; a[8] = u * sw;
  b[0] = 0; b[1] = 0; b[2] = 0; b[3] = -x * sw; b[4] = -y * sw; b[5] = -sw;
  b[6] = x * v * sw; b[7] = y * v * sw; b[8] = v * sw;
}

// Cyclic Jacobi on a symmetric 9x9 (src/linalg.cpp:128-172), then the eigenvector of
// the smallest eigenvalue (first minimum, :174-181) normalised by its last entry
// (:199-202). Returns false when that entry is ~0.
__host__ __device__ inline bool smallest_normalised(const double* m, double* H) {
  constexpr int n = 9;
  double a[n * n], vec[n * n];
  for (int i = 0; i < n * n; ++i) {
    a[i] = m[i];
    vec[i] = (i / n == i % n) ? 1.0 : 0.0;
  }
  for (int sweep = 0; sweep < 100; ++sweep) {
    double off = 0;
    for (int p = 0; p < n; ++p)
      for (int q = p + 1; q < n; ++q) off += a[p * n + q] * a[p * n + q];
    if (off < 1e-30) break;
    for (int p = 0; p < n; ++p)
      for (int q = p + 1; q < n; ++q) {
        const double apq = a[p * n + q];
        if (fabs(apq) < 1e-300) continue;
        const double theta = (a[q * n + q] - a[p * n + p]) / (2.0 * apq);
        double t = sgn(theta) / (fabs(theta) + sqrt(theta * theta + 1.0));
        if (theta == 0.0) t = 1.0;
        const double c = 1.0 / sqrt(t * t + 1.0), s = t * c;
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
  int k = 0;
  for (int i = 1; i < n; ++i)
    if (a[i * n + i] < a[k * n + k]) k = i;
  const double h8 = vec[8 * n + k];
  if (fabs(h8) < 1e-300) return false;
  const double inv = 1.0 / h8;
  for (int i = 0; i < n; ++i) H[i] = vec[i * n + k] * inv;
  return true;
}

// ------------------------------------------------------------ kernels
struct RayView {
  const float* base;  // rays + view * Hy * Wx
  size_t plane;       // n_views * Hy * Wx (channel stride)
};

// Ray cloud (src/ray_pose.cpp:11-59): z-normalised direction, masked weight, and the
// radix key of the weight (descending; +0 for -0) with the point index as payload.
__global__ void k_cloud(RayView r, int N, double2* __restrict__ dst, double* __restrict__ w,
                        uint32_t* __restrict__ keys, int* __restrict__ vals) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const float fx = r.base[n], fy = r.base[r.plane + n], fz = r.base[2 * r.plane + n];
  const float fc = r.base[6 * r.plane + n];
  const double dz = fz;
  const bool ok = fabs(dz) > kZThr;
  double tx = fx, ty = fy;
  if (ok) {
    tx = static_cast<double>(fx) / dz;
    ty = static_cast<double>(fy) / dz;
  }
  dst[n] = make_double2(tx, ty);
  w[n] = ok ? static_cast<double>(fc) : 0.0;
  uint32_t u = ok ? __float_as_uint(fc) : 0u;
  if ((u & 0x7fffffffu) == 0) u = 0;  // -0 sorts with +0, as the reference's comparison does
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  keys[n] = ~u;
  vals[n] = n;
}

// Stable LSD radix sort, 8 bits a pass: per-block digit histograms (digit-major),
// one exclusive scan, then a stable scatter (rounds of 256 consecutive items; rank
// within a warp by match, across warps by a per-digit prefix).
__global__ void k_radix_hist(const uint32_t* __restrict__ keys, int N, int shift, int nb, int* __restrict__ hist) {
  __shared__ int h[256];
  h[threadIdx.x] = 0;
  __syncthreads();
  const int base = blockIdx.x * kTile;
  for (int r = 0; r < kTile / 256; ++r) {
    const int i = base + r * 256 + threadIdx.x;
    if (i < N) atomicAdd(&h[(keys[i] >> shift) & 255], 1);
  }
  __syncthreads();
  hist[threadIdx.x * nb + blockIdx.x] = h[threadIdx.x];
}

__global__ void k_radix_scan(int* __restrict__ hist, int total) {
  __shared__ int warp_sums[32];
  const int t = threadIdx.x, per = (total + 1023) / 1024;
  const int b = t * per, e = min(total, b + per);
  int local = 0;
  for (int i = b; i < e; ++i) local += hist[i];
  int incl = local;
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if ((t & 31) >= o) incl += v;
  }
  if ((t & 31) == 31) warp_sums[t >> 5] = incl;
  __syncthreads();
  if (t < 32) {
    int s = warp_sums[t];
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, s, o);
      if (t >= o) s += v;
    }
    warp_sums[t] = s;
  }
  __syncthreads();
  int run = incl - local + ((t >> 5) ? warp_sums[(t >> 5) - 1] : 0);
  for (int i = b; i < e; ++i) {
    const int v = hist[i];
    hist[i] = run;
    run += v;
  }
}

__global__ void k_radix_scatter(const uint32_t* __restrict__ kin, const int* __restrict__ vin, int N, int shift,
                                int nb, const int* __restrict__ start, uint32_t* __restrict__ kout,
                                int* __restrict__ vout) {
  __shared__ int cnt[8][256];
  __shared__ int base_w[8][256];
  __shared__ int run[256];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  run[t] = start[t * nb + blockIdx.x];
  const int tile = blockIdx.x * kTile;
  for (int r = 0; r < kTile / 256; ++r) {
    const int i = tile + r * 256 + t;
    const bool valid = i < N;
    const uint32_t key = valid ? kin[i] : 0u;
    const int digit = valid ? static_cast<int>((key >> shift) & 255) : 256;
    for (int k = 0; k < 8; ++k) cnt[k][t] = 0;
    __syncthreads();
    const unsigned peers = __match_any_sync(0xffffffffu, digit);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (valid && rank == 0) cnt[warp][digit] = __popc(peers);
    __syncthreads();
    int acc = run[t];
    for (int k = 0; k < 8; ++k) {
      base_w[k][t] = acc;
      acc += cnt[k][t];
    }
    run[t] = acc;
    __syncthreads();
    if (valid) {
      const int pos = base_w[warp][digit] + rank;
      kout[pos] = key;
      vout[pos] = vin[i];
    }
    __syncthreads();
  }
}

// One hypothesis per thread: the 8 drawn candidates' weighted DLT fit
// (src/ray_pose.cpp:61-74, :153-158).
__global__ void k_fit(const int* __restrict__ draws, const int* __restrict__ order, const double2* __restrict__ dst,
                      const double* __restrict__ w, int Hy, int Wx, double* __restrict__ H, int* __restrict__ ok) {
  const int it = threadIdx.x;
  if (it >= kIter) return;
  double ata[81];
  for (int e = 0; e < 81; ++e) ata[e] = 0;
  for (int k = 0; k < kPick; ++k) {
    const int n = order[draws[it * kPick + k]];
    const double2 d = dst[n];
    double a[9], b[9];
    dlt_rows(plane(n % Wx, Wx), plane(n / Wx, Hy), d.x, d.y, w[n], a, b);
    for (int i = 0; i < 9; ++i)
      for (int j = 0; j < 9; ++j) ata[i * 9 + j] += a[i] * a[j] + b[i] * b[j];
  }
  ok[it] = smallest_normalised(ata, H + it * 9) ? 1 : 0;
}

// Inlier masks of every fitted hypothesis over every point (src/ray_pose.cpp:77-93).
__global__ void k_score(const double* __restrict__ H, const int* __restrict__ ok, const double2* __restrict__ dst,
                        int Hy, int Wx, uint8_t* __restrict__ mask) {
  const int it = blockIdx.y;
  if (!ok[it]) return;
  const int N = Hy * Wx;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const double* h = H + it * 9;
  const double x = plane(n % Wx, Wx), y = plane(n / Wx, Hy);
  const double px = h[0] * x + h[1] * y + h[2];
  const double py = h[3] * x + h[4] * y + h[5];
  const double pz = h[6] * x + h[7] * y + h[8];
  const double2 d = dst[n];
  const double ex = px / pz - d.x, ey = py / pz - d.y;
  mask[static_cast<size_t>(it) * N + n] = (ex * ex + ey * ey) < kThr * kThr ? 1 : 0;
}

// Ordered sums, one accumulator per thread in point order as the reference adds them:
// threads 0..99 the inlier weight of each hypothesis (src/ray_pose.cpp:89-91), threads
// 100..102 the confidence-weighted origin and 103 the confidence total (:212-219).
__global__ void k_sums(const uint8_t* __restrict__ mask, const int* __restrict__ ok, const double* __restrict__ w,
                       RayView r, int N, double* __restrict__ scores, double* __restrict__ sums) {
  const int t = threadIdx.x;
  if (t < kIter) {
    if (!ok[t]) return;
    const uint8_t* m = mask + static_cast<size_t>(t) * N;
    double total = 0.0;
    for (int n = 0; n < N; ++n)
      if (m[n]) total += w[n];
    scores[t] = total;
  } else if (t < kIter + 4) {
    const int c = t - kIter;
    const float* conf = r.base + 6 * r.plane;
    double acc = 0.0;
    if (c < 3) {
      const float* o = r.base + (3 + c) * r.plane;
      for (int n = 0; n < N; ++n) acc += static_cast<double>(o[n]) * static_cast<double>(conf[n]);
    } else {
      for (int n = 0; n < N; ++n) acc += static_cast<double>(conf[n]);
    }
    sums[c] = acc;
  }
}

// Best hypothesis: first strictly larger score, starting from -1 (src/ray_pose.cpp:160-164);
// then its mask row.
__global__ void k_pick(const double* __restrict__ scores, const int* __restrict__ ok, int* __restrict__ best) {
  if (threadIdx.x != 0) return;
  double b = -1.0;
  int bi = -1;
  for (int it = 0; it < kIter; ++it)
    if (ok[it] && scores[it] > b) {
      b = scores[it];
      bi = it;
    }
  *best = bi;
}

__global__ void k_best_mask(const uint8_t* __restrict__ mask, const int* __restrict__ best, int N,
                            uint8_t* __restrict__ out) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const int bi = *best;
  out[n] = bi >= 0 ? mask[static_cast<size_t>(bi) * N + n] : 0;
}

// Refit normal matrix: one entry per thread, accumulated over the refit points in
// order (src/linalg.cpp:187-197).
__global__ void k_ata(const int* __restrict__ idx, int M, const double2* __restrict__ dst, const double* __restrict__ w,
                      int Hy, int Wx, double* __restrict__ ata) {
  const int e = threadIdx.x;
  if (e >= 81) return;
  const int i = e / 9, j = e % 9;
  double acc = 0;
  for (int m = 0; m < M; ++m) {
    const int n = idx[m];
    const double2 d = dst[n];
    double a[9], b[9];
    dlt_rows(plane(n % Wx, Wx), plane(n / Wx, Hy), d.x, d.y, w[n], a, b);
    acc += a[i] * a[j] + b[i] * b[j];
  }
  ata[e] = acc;
}

// Householder QR with n-1 reflectors (src/linalg.cpp:45-90), host.
void qr3(const double* a, double* q, double* r) {
  constexpr int n = 3;
  for (int i = 0; i < n * n; ++i) {
    r[i] = a[i];
    q[i] = (i / n == i % n) ? 1.0 : 0.0;
  }
  double v[n];
  for (int k = 0; k + 1 < n; ++k) {
    double nx = 0;
    for (int i = k; i < n; ++i) nx += r[i * n + k] * r[i * n + k];
    nx = sqrt(nx);
    if (nx < 1e-300) continue;
    const double alpha = r[k * n + k] >= 0.0 ? -nx : nx;
    for (int i = 0; i < n; ++i) v[i] = i >= k ? r[i * n + k] : 0.0;
    v[k] -= alpha;
    double vv = 0;
    for (int i = k; i < n; ++i) vv += v[i] * v[i];
    if (vv < 1e-300) continue;
    for (int j = 0; j < n; ++j) {
      double d = 0;
      for (int i = k; i < n; ++i) d += v[i] * r[i * n + j];
      const double f = 2.0 * d / vv;
      for (int i = k; i < n; ++i) r[i * n + j] -= f * v[i];
    }
    for (int row = 0; row < n; ++row) {
      double d = 0;
      for (int i = k; i < n; ++i) d += q[row * n + i] * v[i];
      const double f = 2.0 * d / vv;
      for (int i = k; i < n; ++i) q[row * n + i] -= f * v[i];
    }
  }
  for (int i = 0; i < n; ++i)
    for (int j = 0; j < i; ++j) r[i * n + j] = 0.0;
}

template <typename T>
bool grow(T*& p, size_t count, bool pinned) {
  if (p) {
    if (pinned) cudaFreeHost(p);
    else cudaFree(p);
    p = nullptr;
  }
  void* q = nullptr;
  const cudaError_t e = pinned ? cudaMallocHost(&q, count * sizeof(T)) : cudaMalloc(&q, count * sizeof(T));
  if (e != cudaSuccess) return false;
  p = static_cast<T*>(q);
  return true;
}

template <typename T>
void drop(T*& p, bool pinned) {
  if (!p) return;
  if (pinned) cudaFreeHost(p);
  else cudaFree(p);
  p = nullptr;
}

}  // namespace

double det3(const double a[9]) {  // src/linalg.cpp:10-14
  return a[0] * (a[4] * a[8] - a[5] * a[7]) - a[1] * (a[3] * a[8] - a[5] * a[6]) + a[2] * (a[3] * a[7] - a[4] * a[6]);
}

// QL via the QR of the column-reversed matrix, diag(L) >= 0 (src/linalg.cpp:96-126).
void ql3(const double a[9], double q[9], double l[9]) {
  double ar[9], qq[9], rr[9];
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) ar[i * 3 + j] = a[i * 3 + 2 - j];
  qr3(ar, qq, rr);
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      q[i * 3 + j] = qq[i * 3 + 2 - j];
      l[i * 3 + j] = rr[(2 - i) * 3 + 2 - j];
    }
  const double s[3] = {sgn(l[0]), sgn(l[4]), sgn(l[8])};
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      q[i * 3 + j] *= s[j];
      l[i * 3 + j] *= s[i];
    }
}

RaySolver::~RaySolver() { release(); }

void RaySolver::release() {
  drop(dst_, false);
  drop(w_, false);
  drop(H_, false);
  drop(scores_, false);
  drop(sums_, false);
  drop(ata_, false);
  drop(keys_[0], false);
  drop(keys_[1], false);
  drop(hist_, false);
  drop(vals_[0], false);
  drop(vals_[1], false);
  drop(draws_, false);
  drop(fit_ok_, false);
  drop(best_, false);
  drop(refit_, false);
  drop(mask_, false);
  drop(bestmask_, false);
  drop(h_order_, true);
  drop(h_mask_, true);
  drop(h_small_, true);
  drop(h_refit_, true);
  drop(h_ata_, true);
  cap_ = 0;
  draws_for_ = -1;
}

bool RaySolver::reserve(int N, std::string* err) {
  if (N <= cap_) return true;
  release();
  const size_t n = static_cast<size_t>(N), nb = (n + kTile - 1) / kTile;
  // mask_ holds one byte per (hypothesis, point)
  bool ok = grow(dst_, n, false) && grow(w_, n, false) && grow(H_, static_cast<size_t>(kIter) * 9, false) &&
            grow(scores_, kIter, false) && grow(sums_, 4, false) && grow(ata_, 81, false) &&
            grow(keys_[0], n, false) && grow(keys_[1], n, false) && grow(hist_, 256 * nb, false) &&
            grow(vals_[0], n, false) && grow(vals_[1], n, false) &&
            grow(draws_, static_cast<size_t>(kIter) * kPick, false) && grow(fit_ok_, kIter, false) &&
            grow(best_, 1, false) && grow(refit_, kMaxRefit, false) &&
            grow(mask_, static_cast<size_t>(kIter) * n, false) && grow(bestmask_, n, false) &&
            grow(h_order_, n, true) && grow(h_mask_, n, true) && grow(h_small_, 8, true) &&
            grow(h_refit_, kMaxRefit, true) && grow(h_ata_, 81, true);
  if (!ok) {
    release();
    if (err) *err = "ray pose: out of memory";
    return false;
  }
  cap_ = N;
  return true;
}

int RaySolver::solve(const float* rays, int n_views, int view, int Hy, int Wx, int img_h, int img_w, cudaStream_t s,
                     RayPoseResult* out, std::string* err) {
  const int N = Hy * Wx;
  if (!rays || !out || n_views <= 0 || view < 0 || view >= n_views || Hy <= 0 || Wx <= 0 || N < kPick) {
    if (err) *err = "ray pose: bad arguments (need at least 8 ray points)";
    return -1;
  }
  if (!reserve(N, err)) return -2;
  const int n_cand = std::min(N, std::max(kPick, static_cast<int>(static_cast<double>(N) * kRatio)));
  if (draws_for_ != n_cand) {
    // seeded candidate draws (src/ray_pose.cpp:129-145): one permutation of the pool,
    // partially re-shuffled each iteration; depends on the pool size only
    std::vector<int> draws(static_cast<size_t>(kIter) * kPick), perm(n_cand);
    std::iota(perm.begin(), perm.end(), 0);
    std::mt19937 gen(kSeed);
    for (int it = 0; it < kIter; ++it)
      for (int k = 0; k < kPick; ++k) {
        std::uniform_int_distribution<int> pick(k, n_cand - 1);
        std::swap(perm[k], perm[pick(gen)]);
        draws[static_cast<size_t>(it) * kPick + k] = perm[k];
      }
    if (cudaMemcpy(draws_, draws.data(), draws.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
      if (err) *err = "ray pose: draw upload failed";
      return -3;
    }
    draws_for_ = n_cand;
  }
  const RayView rv{rays + static_cast<size_t>(view) * N, static_cast<size_t>(n_views) * N};
  const int gb = (N + 255) / 256, nb = (N + kTile - 1) / kTile;
  k_cloud<<<gb, 256, 0, s>>>(rv, N, dst_, w_, keys_[0], vals_[0]);
  for (int pass = 0; pass < 4; ++pass) {
    const int src = pass & 1, shift = 8 * pass;
    k_radix_hist<<<nb, 256, 0, s>>>(keys_[src], N, shift, nb, hist_);
    k_radix_scan<<<1, 1024, 0, s>>>(hist_, 256 * nb);
    k_radix_scatter<<<nb, 256, 0, s>>>(keys_[src], vals_[src], N, shift, nb, hist_, keys_[src ^ 1], vals_[src ^ 1]);
  }
  const int* order = vals_[0];  // four passes: back in buffer 0
  const double2* dst = dst_;
  k_fit<<<1, 128, 0, s>>>(draws_, order, dst, w_, Hy, Wx, H_, fit_ok_);
  k_score<<<dim3(gb, kIter), 256, 0, s>>>(H_, fit_ok_, dst, Hy, Wx, mask_);
  k_sums<<<1, 128, 0, s>>>(mask_, fit_ok_, w_, rv, N, scores_, sums_);
  k_pick<<<1, 32, 0, s>>>(scores_, fit_ok_, best_);
  k_best_mask<<<gb, 256, 0, s>>>(mask_, best_, N, bestmask_);
  if (cudaMemcpyAsync(h_order_, order, static_cast<size_t>(N) * sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyAsync(h_mask_, bestmask_, N, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaMemcpyAsync(h_small_, sums_, 4 * sizeof(double), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    if (err) *err = std::string("ray pose: ") + cudaGetErrorString(cudaGetLastError());
    return -4;
  }
  // best-hypothesis inliers by weight, descending and stable (src/ray_pose.cpp:168-194)
  std::vector<int> inl;
  inl.reserve(N);
  for (int p = 0; p < N; ++p)
    if (h_mask_[h_order_[p]]) inl.push_back(h_order_[p]);
  out->n_inlier_best = static_cast<int>(inl.size());
  if (static_cast<int>(inl.size()) > kMaxRefit) {
    const int keep = std::max(static_cast<int>(static_cast<double>(inl.size()) * 0.95), kMaxRefit);
    inl.resize(keep);
    std::mt19937 gen(kSeed ^ 0x9e3779b9u);
    std::shuffle(inl.begin(), inl.end(), gen);
    inl.resize(kMaxRefit);
  }
  if (inl.size() < 4) return 1;
  const int M = static_cast<int>(inl.size());
  memcpy(h_refit_, inl.data(), M * sizeof(int));
  if (cudaMemcpyAsync(refit_, h_refit_, M * sizeof(int), cudaMemcpyHostToDevice, s) != cudaSuccess) {
    if (err) *err = "ray pose: refit upload failed";
    return -5;
  }
  k_ata<<<1, 96, 0, s>>>(refit_, M, dst, w_, Hy, Wx, ata_);
  if (cudaMemcpyAsync(h_ata_, ata_, 81 * sizeof(double), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    if (err) *err = std::string("ray pose: ") + cudaGetErrorString(cudaGetLastError());
    return -6;
  }
  // refit, sign, QL and the pose (src/ray_pose.cpp:197-249)
  double A[9];
  if (!smallest_normalised(h_ata_, A)) return 1;
  if (det3(A) < 0)
    for (double& a : A) a = -a;
  double R[9], L[9];
  ql3(A, R, L);
  const double l22 = L[8];
  if (fabs(l22) < 1e-12) return 1;
  for (double& v : L) v /= l22;
  const double f0 = L[0], f1 = L[4];
  if (fabs(f0) < 1e-12 || fabs(f1) < 1e-12) return 1;
  const double cs = h_small_[3];
  if (fabs(cs) < 1e-12) return 1;
  const double T[3] = {h_small_[0] / cs, h_small_[1] / cs, h_small_[2] / cs};
  memcpy(out->A, A, sizeof(A));
  memcpy(out->R, R, sizeof(R));
  memcpy(out->T, T, sizeof(T));
  out->focal[0] = 1.0 / f0;
  out->focal[1] = 1.0 / f1;
  out->pp[0] = L[6] + 1.0;
  out->pp[1] = L[7] + 1.0;
  for (int i = 0; i < 3; ++i) {
    for (int c = 0; c < 3; ++c) out->ext[i * 4 + c] = static_cast<float>(R[c * 3 + i]);
    out->ext[i * 4 + 3] = static_cast<float>(-(R[0 * 3 + i] * T[0] + R[1 * 3 + i] * T[1] + R[2 * 3 + i] * T[2]));
  }
  for (float& v : out->intr) v = 0.0f;
  out->intr[0] = static_cast<float>(out->focal[0] / 2.0 * img_w);
  out->intr[4] = static_cast<float>(out->focal[1] / 2.0 * img_h);
  out->intr[2] = static_cast<float>(out->pp[0] * img_w * 0.5);
  out->intr[5] = static_cast<float>(out->pp[1] * img_h * 0.5);
  out->intr[8] = 1.0f;
  for (float v : out->ext)
    if (!isfinite(v)) return 1;
  for (float v : out->intr)
    if (!isfinite(v)) return 1;
  return 0;
}

}  // namespace da3b
