// Codec kernels around the k-means core: spherical flip and scales, label
// scatter, bf16 packing, SSVQ fold, int-N quantisation, the streaming
// multi-codebook reconstruction and the least-squares scale re-fit
// (skcq/codebook/{spherical,euclidean,ssvq,aqlm}.py).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace skcq {

__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

inline int grid1d(int64_t work, int threads = 256) {
  int64_t g = (work + threads - 1) / threads;
  if (g > 148 * 32) g = 148 * 32;
  return (int)(g < 1 ? 1 : g);
}

#define GRID_STRIDE(t, total) \
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < (total); t += (int64_t)gridDim.x * blockDim.x)

__global__ void flip_check_kernel(const float* __restrict__ R, const float* __restrict__ C,
                                  const int32_t* __restrict__ labels, int nblk, int n_pad, int k_pad, int bs,
                                  const int32_t* __restrict__ n, unsigned long long* __restrict__ flags) {
  GRID_STRIDE(t, (int64_t)nblk * n_pad) {
    const int64_t b = t / n_pad, i = t % n_pad;
    if (i >= n[b]) continue;
    const int l = labels[t];
    const float* x = R + t * bs;
    const float* c = C + (b * k_pad + l) * bs;
    float s = 0.f;
    for (int j = 0; j < bs; ++j) s = __fmaf_rn(x[j], c[j], s);
    if (s < 0.f) atomicOr(&flags[b], (l < bs && l < 63) ? (1ull << l) : (1ull << 63));
  }
}

__global__ void apply_flip_kernel(const unsigned long long* __restrict__ flags, int nblk, int k_pad, int bs,
                                  float* __restrict__ C) {
  GRID_STRIDE(t, (int64_t)nblk * k_pad * bs) {
    const int64_t j = t % bs, b = t / ((int64_t)k_pad * bs);
    if ((flags[b] >> j) & 1ull) C[t] = -C[t];
  }
}

__global__ void scatter_labels_kernel(const int32_t* __restrict__ labels, const int32_t* __restrict__ rowmap,
                                      const int32_t* __restrict__ n, int nblk, int n_pad, int shared, int n_rows,
                                      int n_blocks, int64_t* __restrict__ idxs) {
  GRID_STRIDE(t, (int64_t)nblk * n_pad) {
    const int64_t b = t / n_pad, i = t % n_pad;
    if (i >= n[b]) continue;
    const int64_t p = rowmap[t];
    int64_t r, bb;
    if (shared) {
      r = p / n_blocks;
      bb = p % n_blocks;
    } else {
      r = p;
      bb = b;
    }
    idxs[bb * n_rows + r] = labels[t];
  }
}

// One warp per row: ||row|| < thr (aqlm.py:146-147, spherical.py:150-151).
__global__ void row_zero_kernel(const float* __restrict__ W, int64_t ld, int n_rows, int in_dim, float thr,
                                uint8_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; r < n_rows;
       r += ((int64_t)gridDim.x * blockDim.x) >> 5) {
    float s = 0.f;
    for (int c = lane; c < in_dim; c += 32) {
      const float v = W[r * ld + c];
      s = __fmaf_rn(v, v, s);
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[r] = sqrtf(s) < thr ? 1 : 0;
  }
}

__global__ void spherical_scales_kernel(const float* __restrict__ W, int64_t ld, int n_rows, int bs, int n_blocks,
                                        int shared, const float* __restrict__ C, int k_pad,
                                        const int64_t* __restrict__ idxs, const uint8_t* __restrict__ row_zero,
                                        float* __restrict__ scales) {
  GRID_STRIDE(t, (int64_t)n_rows * n_blocks) {
    const int64_t r = t / n_blocks, b = t % n_blocks;
    float s = 0.f;
    if (!row_zero[r]) {
      const int64_t idx = idxs[b * n_rows + r];
      const float* c = C + ((shared ? 0 : b) * (int64_t)k_pad + idx) * bs;
      const float* x = W + r * ld + b * bs;
      for (int j = 0; j < bs; ++j) s = __fmaf_rn(x[j], c[j], s);
    }
    scales[t] = s;
  }
}

__global__ void centroids_to_bf16_kernel(const float* __restrict__ C, int nblk, int k_pad, int bs, int K,
                                         uint16_t* __restrict__ out) {
  GRID_STRIDE(t, (int64_t)nblk * bs * K) {
    const int64_t c = t % K, j = (t / K) % bs, b = t / ((int64_t)K * bs);
    out[t] = f32_to_bf16(C[(b * k_pad + c) * bs + j]);
  }
}

__global__ void copy_remainder_kernel(const float* __restrict__ W, int64_t ld, int n_rows, int col0, int rem,
                                      uint16_t* __restrict__ out) {
  GRID_STRIDE(t, (int64_t)n_rows * rem) {
    const int64_t r = t / rem, c = t % rem;
    out[t] = f32_to_bf16(W[r * ld + col0 + c]);
  }
}

__global__ void ssvq_fold_kernel(const void* __restrict__ W, int w_is_bf16, int64_t ld, int n_rows, int in_dim,
                                 float* __restrict__ folded, int8_t* __restrict__ signs,
                                 uint32_t* __restrict__ packed) {
  const int words = (in_dim + 31) / 32;
  GRID_STRIDE(t, (int64_t)n_rows * words) {
    const int64_t r = t / words, w = t % words;
    uint32_t bits = 0;
    const int c0 = (int)w * 32, c1 = min(in_dim, c0 + 32);
    for (int c = c0; c < c1; ++c) {
      const float v = w_is_bf16 ? bf16_to_f32(static_cast<const uint16_t*>(W)[r * ld + c])
                                : static_cast<const float*>(W)[r * ld + c];
      const bool neg = v < 0.f;  // torch.sign(0) == 0 -> +1
      folded[r * in_dim + c] = neg ? -v : v;
      if (signs) signs[r * in_dim + c] = neg ? -1 : 1;
      bits |= (uint32_t)neg << (c - c0);
    }
    if (packed) packed[t] = bits;
  }
}

// One thread per centroid index: column max over all (block, dim) rows, then
// the fake-quantised column (spherical.py:309-315).
__global__ void quantize_centroids_kernel(uint16_t* __restrict__ cb, int rows, int K, int bits) {
  const float levels = (float)((1 << (bits - 1)) - 1);
  GRID_STRIDE(c, (int64_t)K) {
    float m = 0.f;
    for (int r = 0; r < rows; ++r) m = fmaxf(m, fabsf(bf16_to_f32(cb[(int64_t)r * K + c])));
    const float qs = __fdiv_rn(fmaxf(m, 1e-10f), levels);
    for (int r = 0; r < rows; ++r) {
      const float v = bf16_to_f32(cb[(int64_t)r * K + c]);
      float q = rintf(__fdiv_rn(v, qs));
      q = fminf(fmaxf(q, -levels), levels);
      cb[(int64_t)r * K + c] = f32_to_bf16(__fmul_rn(q, qs));
    }
  }
}

__global__ void absmax_kernel(const float* __restrict__ x, int64_t count, unsigned int* __restrict__ out) {
  float m = 0.f;
  GRID_STRIDE(t, count) m = fmaxf(m, fabsf(x[t]));
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));  // non-negative floats order as uints
}

__global__ void quantize_scales_kernel(const float* __restrict__ x, int64_t count, int bits,
                                       const unsigned int* __restrict__ absmax, void* __restrict__ out) {
  const float levels = (float)((1 << (bits - 1)) - 1);
  const float am = __uint_as_float(*absmax);
  if (am == 0.f) return;
  const float qs = __fdiv_rn(am, levels);
  GRID_STRIDE(t, count) {
    float q = rintf(__fdiv_rn(x[t], qs));
    q = fminf(fmaxf(q, -levels), levels);
    if (bits <= 8)
      static_cast<int8_t*>(out)[t] = (int8_t)q;
    else
      static_cast<int16_t*>(out)[t] = (int16_t)q;
  }
}

__global__ void finish_qscale_kernel(unsigned int* absmax_then_qscale, int bits) {
  const float levels = (float)((1 << (bits - 1)) - 1);
  const float am = __uint_as_float(*absmax_then_qscale);
  *reinterpret_cast<float*>(absmax_then_qscale) = am == 0.f ? 0.f : __fdiv_rn(am, levels);
}

struct CodecSet {
  skcq_codec_desc c[SKCQ_MAX_CODECS];
  int n;
};

__device__ __forceinline__ float load_scale(const skcq_codec_desc& d, int64_t r, int64_t b) {
  const int64_t o = r * d.scale_ld + b;
  switch (d.scale_dtype) {
    case 0: return static_cast<const float*>(d.scales)[o];
    case 1: return bf16_to_f32(static_cast<const uint16_t*>(d.scales)[o]);
    case 2: return __half2float(static_cast<const __half*>(d.scales)[o]);
    case 3: return __fmul_rn((float)static_cast<const int8_t*>(d.scales)[o], d.q_scale);
    default: return __fmul_rn((float)static_cast<const int16_t*>(d.scales)[o], d.q_scale);
  }
}

// Value of one codec's reconstruction at (r, col): spherical.py:205-210,
// euclidean.py:435-439, signs per ssvq.py:62-65.
__device__ __forceinline__ float codec_value(const skcq_codec_desc& d, int64_t r, int col) {
  const int cov = d.n_blocks * d.bs;
  float v;
  if (col < cov) {
    const int b = col / d.bs, j = col - b * d.bs;
    const int64_t idx = d.idxs[(int64_t)b * d.idx_ld + r];
    const int64_t cb = d.shared ? 0 : b;
    v = bf16_to_f32(d.cent_t ? d.cent_t[(cb * d.K + idx) * d.bs + j] : d.cent[(cb * d.bs + j) * d.K + idx]);
    if (d.kind == 0) v = __fmul_rn(load_scale(d, r, b), v);
  } else {
    v = d.rem ? bf16_to_f32(d.rem[r * d.rem_cols + (col - cov)]) : 0.f;
  }
  if (d.signs && col < d.sign_cols) v = __fmul_rn(v, (float)d.signs[r * d.sign_ld + col]);
  return v;
}

// One CTA per (64-row tile, 128-column stripe), row tiles fastest in the
// grid: the CTAs in flight share a column stripe, so the centroid tables of
// the stripe's blocks (for a 128-column stripe of the bs=4 K=65536 table,
// 16 MB instead of the whole 268 MB) stay in L2 while every row gathers from
// them, and each block's int64 indices for the tile's consecutive rows come
// in whole cache lines. Threads walk the tile column-fastest (coalesced raw
// and out). The arithmetic per element is the same fixed codec order as the
// reference's sum.
constexpr int RC_ROWS = 64, RC_COLS = 128, RC_THREADS = 256;

__global__ void __launch_bounds__(RC_THREADS) reconstruct_kernel(CodecSet set, int n_rows, int in_dim,
                                                                 const float* __restrict__ raw, int64_t raw_ld,
                                                                 float* __restrict__ out, int64_t out_ld) {
  const int64_t r0 = (int64_t)blockIdx.x * RC_ROWS;
  const int c0 = blockIdx.y * RC_COLS;
  const int64_t left = (int64_t)n_rows - r0;
  const int rows = left < RC_ROWS ? (int)left : RC_ROWS;
  const int cols = min(RC_COLS, in_dim - c0);
  for (int e = threadIdx.x; e < RC_ROWS * RC_COLS; e += RC_THREADS) {
    const int dr = e / RC_COLS, dc = e % RC_COLS;
    if (dr >= rows || dc >= cols) continue;
    const int64_t r = r0 + dr;
    const int col = c0 + dc;
    float acc = codec_value(set.c[0], r, col);
    for (int i = 1; i < set.n; ++i) acc = __fadd_rn(acc, codec_value(set.c[i], r, col));
    out[r * out_ld + col] = raw ? __fsub_rn(raw[r * raw_ld + col], acc) : acc;
  }
}

// aqlm.py:239-252 for one (row, block).
__global__ void refit_kernel(skcq_codec_desc d, const float* __restrict__ raw, int64_t raw_ld,
                             const float* __restrict__ recon, int64_t recon_ld, int n_rows,
                             const uint8_t* __restrict__ row_zero, float* __restrict__ scales) {
  GRID_STRIDE(t, (int64_t)n_rows * d.n_blocks) {
    const int64_t r = t / d.n_blocks, b = t % d.n_blocks;
    if (row_zero[r]) {
      scales[r * d.scale_ld + b] = 0.f;
      continue;
    }
    const int64_t idx = d.idxs[b * d.idx_ld + r];
    const float so = static_cast<const float*>(d.scales)[r * d.scale_ld + b];
    float dot = 0.f, nn = 0.f;
    for (int j = 0; j < d.bs; ++j) {
      const int col = (int)b * d.bs + j;
      float pd = bf16_to_f32(d.cent[((int64_t)(d.shared ? 0 : b) * d.bs + j) * d.K + idx]);
      if (d.signs) pd = __fmul_rn(pd, (float)d.signs[r * d.sign_ld + col]);
      const float other = __fsub_rn(recon[r * recon_ld + col], __fmul_rn(so, pd));
      const float target = __fsub_rn(raw[r * raw_ld + col], other);
      dot = __fmaf_rn(target, pd, dot);
      nn = __fmaf_rn(pd, pd, nn);
    }
    const float nrm = sqrtf(nn);
    scales[r * d.scale_ld + b] = __fdiv_rn(dot, __fadd_rn(__fmul_rn(nrm, nrm), 1e-10f));
  }
}

}  // namespace skcq

using namespace skcq;

#define LAUNCH_CHECK(name) return check_launch(name)

extern "C" int skcq_flip_check(const float* R, const float* C, const int32_t* labels, int nblk, int n_pad, int k_pad,
                               int bs, const int32_t* n, uint64_t* flags, void* stream) {
  SKCQ_REQUIRE(R && C && labels && n && flags, SKCQ_ERR_INVALID, "flip_check: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(flags, 0, sizeof(uint64_t) * nblk, s);
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "flip_check: %s", cudaGetErrorString(e));
  flip_check_kernel<<<grid1d((int64_t)nblk * n_pad), 256, 0, s>>>(R, C, labels, nblk, n_pad, k_pad, bs, n,
                                                                    (unsigned long long*)flags);
  LAUNCH_CHECK("flip_check");
}

extern "C" int skcq_apply_flip(const uint64_t* flags, int nblk, int k_pad, int bs, float* C, void* stream) {
  SKCQ_REQUIRE(flags && C, SKCQ_ERR_INVALID, "apply_flip: null pointer");
  SKCQ_REQUIRE(bs < 64, SKCQ_ERR_INVALID, "apply_flip: block size %d >= 64", bs);
  apply_flip_kernel<<<grid1d((int64_t)nblk * k_pad * bs), 256, 0, (cudaStream_t)stream>>>(
      (const unsigned long long*)flags, nblk, k_pad, bs, C);
  LAUNCH_CHECK("apply_flip");
}

extern "C" int skcq_scatter_labels(const int32_t* labels, const int32_t* rowmap, const int32_t* n, int nblk,
                                   int n_pad, int shared, int n_rows, int n_blocks, int64_t* idxs, void* stream) {
  SKCQ_REQUIRE(labels && rowmap && n && idxs, SKCQ_ERR_INVALID, "scatter_labels: null pointer");
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(idxs, 0, sizeof(int64_t) * (size_t)n_rows * n_blocks, s);
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "scatter_labels: %s", cudaGetErrorString(e));
  scatter_labels_kernel<<<grid1d((int64_t)nblk * n_pad), 256, 0, s>>>(labels, rowmap, n, nblk, n_pad, shared, n_rows,
                                                                        n_blocks, idxs);
  LAUNCH_CHECK("scatter_labels");
}

extern "C" int skcq_row_zero_mask(const float* W, int64_t ld, int n_rows, int in_dim, float thr, uint8_t* out,
                                  void* stream) {
  SKCQ_REQUIRE(W && out, SKCQ_ERR_INVALID, "row_zero_mask: null pointer");
  row_zero_kernel<<<grid1d((int64_t)n_rows * 32), 256, 0, (cudaStream_t)stream>>>(W, ld, n_rows, in_dim, thr, out);
  LAUNCH_CHECK("row_zero_mask");
}

extern "C" int skcq_spherical_scales(const float* W, int64_t ld, int n_rows, int bs, int n_blocks, int shared,
                                     const float* C, int k_pad, const int64_t* idxs, const uint8_t* row_zero,
                                     float* scales, void* stream) {
  SKCQ_REQUIRE(W && C && idxs && row_zero && scales, SKCQ_ERR_INVALID, "spherical_scales: null pointer");
  spherical_scales_kernel<<<grid1d((int64_t)n_rows * n_blocks), 256, 0, (cudaStream_t)stream>>>(
      W, ld, n_rows, bs, n_blocks, shared, C, k_pad, idxs, row_zero, scales);
  LAUNCH_CHECK("spherical_scales");
}

extern "C" int skcq_centroids_to_bf16(const float* C, int nblk, int k_pad, int bs, int K, uint16_t* out,
                                      void* stream) {
  SKCQ_REQUIRE(C && out && K <= k_pad, SKCQ_ERR_INVALID, "centroids_to_bf16: bad arguments");
  centroids_to_bf16_kernel<<<grid1d((int64_t)nblk * bs * K), 256, 0, (cudaStream_t)stream>>>(C, nblk, k_pad, bs, K,
                                                                                             out);
  LAUNCH_CHECK("centroids_to_bf16");
}

extern "C" int skcq_copy_remainder(const float* W, int64_t ld, int n_rows, int col0, int rem, uint16_t* out,
                                   void* stream) {
  SKCQ_REQUIRE(W && out, SKCQ_ERR_INVALID, "copy_remainder: null pointer");
  if (rem <= 0 || n_rows <= 0) return SKCQ_OK;
  copy_remainder_kernel<<<grid1d((int64_t)n_rows * rem), 256, 0, (cudaStream_t)stream>>>(W, ld, n_rows, col0, rem,
                                                                                        out);
  LAUNCH_CHECK("copy_remainder");
}

extern "C" int skcq_ssvq_fold(const void* W, int w_is_bf16, int64_t ld, int n_rows, int in_dim, float* folded,
                              int8_t* signs, uint32_t* packed, void* stream) {
  SKCQ_REQUIRE(W && folded, SKCQ_ERR_INVALID, "ssvq_fold: null pointer");
  if (n_rows <= 0 || in_dim <= 0) return SKCQ_OK;
  const int64_t work = (int64_t)n_rows * ((in_dim + 31) / 32);
  ssvq_fold_kernel<<<grid1d(work), 256, 0, (cudaStream_t)stream>>>(W, w_is_bf16, ld, n_rows, in_dim, folded, signs,
                                                                   packed);
  LAUNCH_CHECK("ssvq_fold");
}

extern "C" int skcq_quantize_centroids(uint16_t* cb, int rows, int K, int bits, void* stream) {
  SKCQ_REQUIRE(cb, SKCQ_ERR_INVALID, "quantize_centroids: null pointer");
  SKCQ_REQUIRE(bits >= 2 && bits <= 16, SKCQ_ERR_INVALID, "quantize_centroids: bits %d outside [2, 16]", bits);
  if (bits >= 16) return SKCQ_OK;
  quantize_centroids_kernel<<<grid1d(K, 128), 128, 0, (cudaStream_t)stream>>>(cb, rows, K, bits);
  LAUNCH_CHECK("quantize_centroids");
}

extern "C" int skcq_quantize_scales(const float* scales, int64_t count, int bits, void* out, float* q_scale_out,
                                    void* stream) {
  SKCQ_REQUIRE(scales && out && q_scale_out, SKCQ_ERR_INVALID, "quantize_scales: null pointer");
  SKCQ_REQUIRE(bits >= 2 && bits <= 16, SKCQ_ERR_INVALID, "quantize_scales: bits %d outside [2, 16]", bits);
  cudaStream_t s = (cudaStream_t)stream;
  unsigned int* word = reinterpret_cast<unsigned int*>(q_scale_out);
  cudaError_t e = cudaMemsetAsync(word, 0, sizeof(unsigned int), s);
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "quantize_scales: %s", cudaGetErrorString(e));
  absmax_kernel<<<grid1d(count), 256, 0, s>>>(scales, count, word);
  quantize_scales_kernel<<<grid1d(count), 256, 0, s>>>(scales, count, bits, word, out);
  finish_qscale_kernel<<<1, 1, 0, s>>>(word, bits);
  LAUNCH_CHECK("quantize_scales");
}

extern "C" int skcq_reconstruct(const skcq_codec_desc* codecs, int n_codecs, int n_rows, int in_dim, const float* raw,
                                int64_t raw_ld, float* out, int64_t out_ld, void* stream) {
  SKCQ_REQUIRE(codecs && out, SKCQ_ERR_INVALID, "reconstruct: null pointer");
  SKCQ_REQUIRE(n_codecs >= 1 && n_codecs <= SKCQ_MAX_CODECS, SKCQ_ERR_INVALID, "reconstruct: %d codecs", n_codecs);
  CodecSet set;
  set.n = n_codecs;
  for (int i = 0; i < n_codecs; ++i) {
    const skcq_codec_desc& d = codecs[i];
    SKCQ_REQUIRE(d.cent && d.idxs && d.bs > 0 && d.n_blocks >= 0, SKCQ_ERR_INVALID, "reconstruct: codec %d", i);
    SKCQ_REQUIRE(d.kind != 0 || d.scales, SKCQ_ERR_INVALID, "reconstruct: spherical codec %d without scales", i);
    SKCQ_REQUIRE(d.n_blocks * d.bs + d.rem_cols == in_dim, SKCQ_ERR_INVALID,
                 "reconstruct: codec %d covers %d + %d columns, expected %d", i, d.n_blocks * d.bs, d.rem_cols, in_dim);
    set.c[i] = d;
  }
  if (n_rows <= 0 || in_dim <= 0) return SKCQ_OK;
  const dim3 grid((unsigned)(((int64_t)n_rows + RC_ROWS - 1) / RC_ROWS), (unsigned)((in_dim + RC_COLS - 1) / RC_COLS));
  SKCQ_REQUIRE(grid.y <= 65535, SKCQ_ERR_INVALID, "reconstruct: in_dim %d too wide", in_dim);
  reconstruct_kernel<<<grid, RC_THREADS, 0, (cudaStream_t)stream>>>(set, n_rows, in_dim, raw, raw_ld, out, out_ld);
  LAUNCH_CHECK("reconstruct");
}

extern "C" int skcq_refit_scales(const skcq_codec_desc* primary, const float* raw, int64_t raw_ld, const float* recon,
                                 int64_t recon_ld, int n_rows, const uint8_t* row_zero, float* scales, void* stream) {
  SKCQ_REQUIRE(primary && raw && recon && row_zero && scales, SKCQ_ERR_INVALID, "refit_scales: null pointer");
  skcq_codec_desc d = *primary;
  SKCQ_REQUIRE(d.kind == 0 && d.scale_dtype == 0, SKCQ_ERR_INVALID, "refit_scales: needs a spherical codec with f32 scales");
  d.scales = scales;
  if (n_rows <= 0 || d.n_blocks <= 0) return SKCQ_OK;
  refit_kernel<<<grid1d((int64_t)n_rows * d.n_blocks), 256, 0, (cudaStream_t)stream>>>(d, raw, raw_ld, recon,
                                                                                       recon_ld, n_rows, row_zero,
                                                                                       scales);
  LAUNCH_CHECK("refit_scales");
}
