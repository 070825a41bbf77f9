// Point and centroid preparation for the batched k-means problem sets:
// zero-block compaction, gather/normalise, split-tf32 operand packing, Forgy
// initialisation (skcq/codebook/spherical.py:243-262, euclidean.py:455-478,
// kmeans.py:142-144 / 201-202).
#include "common.cuh"

namespace skcq {

// Address of element j of source point p of problem b.
__device__ __forceinline__ const float* src_point(const float* W, int64_t ld, int bs, int n_blocks, int shared,
                                                  int b, int64_t p) {
  if (shared) {
    int64_t r = p / n_blocks, bb = p % n_blocks;
    return W + r * ld + bb * (int64_t)bs;
  }
  return W + p * ld + (int64_t)b * bs;
}

// One CTA per problem: ordered compaction of non-zero points.
__global__ void compact_points_kernel(const float* __restrict__ W, int64_t ld, int n_rows, int bs, int n_blocks,
                                      int shared, float thr, int skip_zeros, int n_pad, int32_t* rowmap,
                                      int32_t* n_out) {
  const int b = blockIdx.x;
  const int64_t npts = shared ? (int64_t)n_rows * n_blocks : n_rows;
  int base = 0;
  for (int64_t p0 = 0; p0 < npts; p0 += blockDim.x) {
    int64_t p = p0 + threadIdx.x;
    int keep = 0;
    if (p < npts) {
      if (skip_zeros) {
        const float* x = src_point(W, ld, bs, n_blocks, shared, b, p);
        float s = 0.f;
        for (int j = 0; j < bs; ++j) s = __fmaf_rn(x[j], x[j], s);
        keep = !(sqrtf(s) < thr);
      } else {
        keep = 1;
      }
    }
    int total;
    int pos = block_exclusive_scan(keep, &total);
    if (keep) rowmap[(int64_t)b * n_pad + base + pos] = (int32_t)p;
    base += total;
  }
  if (threadIdx.x == 0) n_out[b] = base;
}

__global__ void gather_points_kernel(const float* __restrict__ W, int64_t ld, int bs, int n_blocks, int shared,
                                     int nblk, const int32_t* __restrict__ rowmap, const int32_t* __restrict__ n,
                                     int n_pad, int normalize, float* __restrict__ X, float* __restrict__ R) {
  const int64_t total = (int64_t)nblk * n_pad;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int b = (int)(t / n_pad);
    const int i = (int)(t % n_pad);
    float* xo = X + t * bs;
    float* ro = R ? R + t * bs : nullptr;
    if (i >= n[b]) {
      for (int j = 0; j < bs; ++j) {
        xo[j] = 0.f;
        if (ro) ro[j] = 0.f;
      }
      continue;
    }
    const float* x = src_point(W, ld, bs, n_blocks, shared, b, rowmap[t]);
    float den = 1.f;
    if (normalize) {
      float s = 0.f;
      for (int j = 0; j < bs; ++j) s = __fmaf_rn(x[j], x[j], s);
      den = fmaxf(sqrtf(s), 1e-12f);
    }
    for (int j = 0; j < bs; ++j) {
      float v = x[j];
      if (ro) ro[j] = v;
      xo[j] = normalize ? __fdiv_rn(v, den) : v;
    }
  }
}

// Split-tf32 operand row: [hi(bs) | lo(bs) | hi(bs) | (l2) 1 1 | 0...] for points,
// [hi | hi | lo | (l2) bhi blo | 0...] for centroids, so that
// A.B = xh.ch + xl.ch + xh.cl (+ bias) ~ x.c to ~2^-21 relative.
__device__ __forceinline__ float packed_value(int metric, bool is_point, const float* v, float bias, int bs,
                                              int kk) {
  const int seg = kk / bs, j = kk - seg * bs;
  if (seg < 3) {
    float hi = tf32_rna(v[j]);
    float lo = tf32_rna(v[j] - hi);
    if (is_point) return seg == 1 ? lo : hi;
    return seg == 2 ? lo : hi;
  }
  const int e = kk - 3 * bs;
  if (metric == SKCQ_METRIC_L2 && e < 2) {
    if (is_point) return 1.0f;
    float bh = tf32_rna(bias);
    return e == 0 ? bh : tf32_rna(bias - bh);
  }
  return 0.f;
}

// Canonical no-swizzle K-major position of element (row, kk) in a
// [rows/8][kp/4][8][4] array.
__device__ __forceinline__ int64_t canon_index(int64_t row, int kk, int kp) {
  return ((row >> 3) * (kp >> 2) + (kk >> 2)) * 32 + (row & 7) * 4 + (kk & 3);
}

__global__ void pack_points_kernel(int metric, const float* __restrict__ X, int nblk, int n_pad, int bs, int kp,
                                   float* __restrict__ A) {
  const int64_t total = (int64_t)nblk * n_pad;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / n_pad, i = t % n_pad;
    float v[64];
    for (int j = 0; j < bs; ++j) v[j] = X[t * bs + j];
    float* dst = A + b * (int64_t)n_pad * kp;
    for (int kk = 0; kk < kp; ++kk) dst[canon_index(i, kk, kp)] = packed_value(metric, true, v, 0.f, bs, kk);
  }
}

__global__ void pack_centroids_kernel(int metric, const float* __restrict__ C, int nblk, int k_pad, int bs, int kp,
                                      const int32_t* __restrict__ k, const int32_t* __restrict__ active,
                                      float* __restrict__ B, float* __restrict__ cnorm) {
  const int64_t total = (int64_t)nblk * k_pad;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / k_pad, c = t % k_pad;
    if (active && !active[b]) continue;
    float v[64];
    float nrm = 0.f;
    const bool valid = c < k[b];
    for (int j = 0; j < bs; ++j) {
      v[j] = valid ? C[t * bs + j] : 0.f;
      nrm = __fmaf_rn(v[j], v[j], nrm);
    }
    cnorm[t] = nrm;
    const float bias = -0.5f * nrm;
    float* dst = B + b * (int64_t)k_pad * kp;
    for (int kk = 0; kk < kp; ++kk) dst[canon_index(c, kk, kp)] = valid ? packed_value(metric, false, v, bias, bs, kk) : 0.f;
  }
}

__global__ void init_from_points_kernel(const float* __restrict__ X, int n_pad, int bs, int nblk,
                                        const int64_t* __restrict__ perm, int64_t perm_ld,
                                        const int32_t* __restrict__ k, int k_pad, float* __restrict__ C) {
  const int64_t total = (int64_t)nblk * k_pad * bs;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t j = t % bs, c = (t / bs) % k_pad, b = t / ((int64_t)bs * k_pad);
    float v = 0.f;
    if (c < k[b]) v = X[(b * n_pad + perm[b * perm_ld + c]) * bs + j];
    C[t] = v;
  }
}

inline int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  if (g > 148 * 16) g = 148 * 16;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace skcq

using namespace skcq;

extern "C" int skcq_compact_points(const float* W, int64_t ld, int n_rows, int bs, int n_blocks, int shared,
                                   float thr, int skip_zeros, int nblk, int npts_pad, int32_t* rowmap,
                                   int32_t* n_out, void* stream) {
  SKCQ_REQUIRE(W && rowmap && n_out, SKCQ_ERR_INVALID, "compact_points: null pointer");
  SKCQ_REQUIRE(bs > 0 && n_rows >= 0 && n_blocks > 0, SKCQ_ERR_INVALID, "compact_points: bad sizes");
  SKCQ_REQUIRE(nblk == (shared ? 1 : n_blocks), SKCQ_ERR_INVALID, "compact_points: nblk must be %d",
               shared ? 1 : n_blocks);
  int64_t npts = shared ? (int64_t)n_rows * n_blocks : n_rows;
  SKCQ_REQUIRE(npts <= npts_pad && npts_pad < (1ll << 31), SKCQ_ERR_INVALID,
               "compact_points: %lld points exceed the padded capacity %d", (long long)npts, npts_pad);
  compact_points_kernel<<<nblk, 1024, 0, (cudaStream_t)stream>>>(W, ld, n_rows, bs, n_blocks, shared, thr,
                                                                 skip_zeros, npts_pad, rowmap, n_out);
  return check_launch("compact_points");
}

extern "C" int skcq_gather_points(const float* W, int64_t ld, int bs, int n_blocks, int shared, int nblk,
                                  const int32_t* rowmap, const int32_t* n, int n_pad, int normalize, float* X,
                                  float* R, void* stream) {
  SKCQ_REQUIRE(W && rowmap && n && X, SKCQ_ERR_INVALID, "gather_points: null pointer");
  SKCQ_REQUIRE(bs > 0 && bs <= 64, SKCQ_ERR_INVALID, "gather_points: block size %d outside [1, 64]", bs);
  int64_t work = (int64_t)nblk * n_pad;
  gather_points_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(W, ld, bs, n_blocks, shared, nblk,
                                                                              rowmap, n, n_pad, normalize, X, R);
  return check_launch("gather_points");
}

extern "C" int skcq_pack_points(int metric, const float* X, int nblk, int n_pad, int bs, float* A, void* stream) {
  SKCQ_REQUIRE(X && A, SKCQ_ERR_INVALID, "pack_points: null pointer");
  SKCQ_REQUIRE(bs > 0 && bs <= 64 && n_pad % 8 == 0, SKCQ_ERR_INVALID, "pack_points: bad sizes");
  int kp = skcq_packed_width(metric, bs);
  int64_t work = (int64_t)nblk * n_pad;
  pack_points_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(metric, X, nblk, n_pad, bs, kp, A);
  return check_launch("pack_points");
}

extern "C" int skcq_pack_centroids(int metric, const float* C, int nblk, int k_pad, int bs, const int32_t* k,
                                   const int32_t* active, float* B, float* cnorm, void* stream) {
  SKCQ_REQUIRE(C && k && B && cnorm, SKCQ_ERR_INVALID, "pack_centroids: null pointer");
  SKCQ_REQUIRE(bs > 0 && bs <= 64 && k_pad % 8 == 0, SKCQ_ERR_INVALID, "pack_centroids: bad sizes");
  int kp = skcq_packed_width(metric, bs);
  int64_t work = (int64_t)nblk * k_pad;
  pack_centroids_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(metric, C, nblk, k_pad, bs, kp, k,
                                                                               active, B, cnorm);
  return check_launch("pack_centroids");
}

extern "C" int skcq_init_from_points(const float* X, int n_pad, int bs, int nblk, const int64_t* perm,
                                     int64_t perm_ld, const int32_t* k, int k_pad, float* C, void* stream) {
  SKCQ_REQUIRE(X && perm && k && C, SKCQ_ERR_INVALID, "init_from_points: null pointer");
  int64_t work = (int64_t)nblk * k_pad * bs;
  init_from_points_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(X, n_pad, bs, nblk, perm, perm_ld,
                                                                                 k, k_pad, C);
  return check_launch("init_from_points");
}
