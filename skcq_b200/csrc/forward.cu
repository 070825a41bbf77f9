// Codebook-expert forward (skcq/codebook_experts.py:30-74 _codebook_pass /
// _remainder_pass, :325-339 CodebookModule.forward, :454-481 CodebookExperts.forward).
//
// Device layout, built once per module from the reference's buffers:
//   table    (n_blocks, K, bs)   centroid vectors contiguous (the reference's
//                                codebook is (n_blocks, bs, K): a gather of one
//                                centroid there touches bs sectors, here one)
//   idx16    (E, n_blocks, out)  uint16 assignments (coalesced over outputs)
//   sign     (E, n_blocks, out)  uint32 bitmask, bit j = column b*bs+j negated
//   scales   (E, n_blocks, out)  as stored (f32 | bf16 | f16 | int8 | int16)
//   remainder(E, out, rem)       as stored (f32 | bf16)
//
// Rows are (token, top-k slot) pairs sorted by expert; a segment is the run of
// rows routed to one expert. One CTA owns (segment, 128 outputs, block range):
// each thread owns one output feature, gathers the expert's centroid for every
// block of its range once per chunk of rows held in shared memory, and
// accumulates in fp32. The block range split ("splits") gives decode enough
// CTAs; split s writes partial sums to slot s of a [splits][rows][out] buffer,
// layers of one module accumulate into the same slots in launch order, and the
// consumer (slot sum, SwiGLU or the weighted combine) adds the slots in a
// fixed order, so results do not depend on scheduling. Splits are the
// slowest-varying grid index so that concurrently running CTAs touch the same
// blocks' tables (L2 reuse of large codebooks).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "fwd_common.cuh"

namespace skcq {

inline int gridf(int64_t work, int threads = 256) {
  int64_t g = (work + threads - 1) / threads;
  if (g > 148 * 32) g = 148 * 32;
  return (int)(g < 1 ? 1 : g);
}

// ---------------------------------------------------------------------------
// Layout preparation
// ---------------------------------------------------------------------------

// out[i] = (uint16) idx[i]; an index outside [0, K) is stored as 0 and flagged.
__global__ void pack_idx16_kernel(const int64_t* __restrict__ src, int64_t n, int K, uint16_t* __restrict__ dst,
                                  int* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t v = src[i];
    if (v < 0 || v >= K) {
      atomicCAS(err, 0, 42);
      v = 0;
    }
    dst[i] = (uint16_t)v;
  }
}

// table[b][k][j] = cb[b][j][k] (element size 2 or 4 bytes). One thread per
// centroid (b, k): its bs reads are each part of a warp-wide read of 32
// consecutive centroids of one coordinate row, and its bs values are written
// as one contiguous run.
template <typename T>
__global__ void transpose_cb_kernel(const T* __restrict__ cb, int64_t nb, int bs, int64_t K, T* __restrict__ table) {
  const int64_t total = nb * K;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / K, k = i - b * K;
    const T* src = cb + b * bs * K + k;
    T* dst = table + i * bs;
    for (int j = 0; j < bs; ++j) dst[j] = src[(int64_t)j * K];
  }
}

// mask[e][b][o] bit j = signs[e][o][b*bs+j] < 0; a sign other than +-1 is flagged.
__global__ void pack_signs_kernel(const int8_t* __restrict__ signs, int E, int out, int64_t ld, int nb, int bs,
                                  uint32_t* __restrict__ mask, int* err) {
  const int64_t total = (int64_t)E * nb * out;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int o = (int)(i % out);
    const int64_t eb = i / out;
    const int b = (int)(eb % nb), e = (int)(eb / nb);
    const int8_t* s = signs + ((int64_t)e * out + o) * ld + (int64_t)b * bs;
    uint32_t m = 0;
    for (int j = 0; j < bs; ++j) {
      const int v = s[j];
      if (v != 1 && v != -1) atomicCAS(err, 0, 43);
      m |= (uint32_t)(v < 0) << j;
    }
    mask[i] = m;
  }
}

// ---------------------------------------------------------------------------
// Routing: stable sort of pairs by expert (codebook_experts.py:462-470)
// ---------------------------------------------------------------------------

constexpr int RT_THREADS = 1024;
constexpr int RT_SMALL_E = 256;  // chunked warp-ranking path up to this many experts

// skip != 0: a negative id marks a slot routed elsewhere (expert-parallel
// receive buffers) and goes to the trailing bucket without an error.
__device__ __forceinline__ int pair_bucket(const int64_t* topk, int T, int k, int E, int p, int* err, int skip) {
  const int kp = p / T, t = p - kp * T;
  const int64_t e = topk[(int64_t)t * k + kp];
  if (e < 0 || e >= E) {
    if (!(skip && e < 0)) atomicCAS(err, 0, 41);
    return E;  // trailing bucket: never computed
  }
  return (int)e;
}

// One CTA. Pair p = kpos * T + token (the order of torch.where(expert_mask[e]):
// kpos-major, then token). perm[pos] = p in (expert, p) order; inv[p] = pos;
// seg[e] = first row of expert e (seg[E] = rows of valid experts);
// active[0] = number of experts with rows, active[1..] their ids ascending.
__global__ void __launch_bounds__(RT_THREADS) route_sort_kernel(const int64_t* __restrict__ topk, int T, int k, int E,
                                                                int32_t* __restrict__ perm, int32_t* __restrict__ seg,
                                                                int32_t* __restrict__ inv, int32_t* __restrict__ active,
                                                                int* err, int skip) {
  extern __shared__ int sm[];
  const int NB = E + 1;  // buckets incl. the invalid one
  int* cnt = sm;         // [NB]
  int* base = sm + NB;   // [NB]
  int* tot = base + NB;  // [NB]
  int* wcnt = tot + NB;  // [32][NB] (small-E path)
  const int P = T * k;
  const int tid = threadIdx.x;
  for (int b = tid; b < NB; b += RT_THREADS) cnt[b] = 0;
  __syncthreads();
  for (int p = tid; p < P; p += RT_THREADS) atomicAdd(&cnt[pair_bucket(topk, T, k, E, p, err, skip)], 1);
  __syncthreads();
  if (tid == 0) {
    int run = 0, na = 0;
    for (int b = 0; b < NB; ++b) {
      base[b] = run;
      if (b < E) {
        seg[b] = run;
        if (cnt[b] > 0) active[1 + na++] = b;
      }
      run += cnt[b];
    }
    seg[E] = base[E];
    active[0] = na;
  }
  __syncthreads();
  if (E <= RT_SMALL_E) {
    const int w = tid >> 5, lane = tid & 31;
    for (int c0 = 0; c0 < P; c0 += RT_THREADS) {
      for (int i = tid; i < 32 * NB; i += RT_THREADS) wcnt[i] = 0;
      __syncthreads();
      const int p = c0 + tid;
      const int bk = p < P ? pair_bucket(topk, T, k, E, p, err, skip) : -1;
      const unsigned peers = __match_any_sync(0xffffffffu, bk);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      if (bk >= 0 && lane == __ffs(peers) - 1) wcnt[w * NB + bk] = __popc(peers);
      __syncthreads();
      for (int b = tid; b < NB; b += RT_THREADS) {
        int run = 0;
        for (int ww = 0; ww < 32; ++ww) {
          const int c = wcnt[ww * NB + b];
          wcnt[ww * NB + b] = run;
          run += c;
        }
        tot[b] = run;
      }
      __syncthreads();
      if (bk >= 0) {
        const int pos = base[bk] + wcnt[w * NB + bk] + rank;
        perm[pos] = p;
        inv[p] = pos;
      }
      __syncthreads();
      for (int b = tid; b < NB; b += RT_THREADS) base[b] += tot[b];
      __syncthreads();
    }
  } else {
    // each bucket's owner thread appends its pairs in ascending order
    for (int b = tid; b < NB; b += RT_THREADS) {
      int pos = base[b];
      for (int p = 0; p < P; ++p) {
        const int kp = p / T, t = p - kp * T;
        const int64_t e = topk[(int64_t)t * k + kp];
        const int bk = (e < 0 || e >= E) ? E : (int)e;
        if (bk == b) {
          perm[pos] = p;
          inv[p] = pos;
          ++pos;
        }
      }
    }
  }
}

// Multi-CTA form for large batches (up to RT_SMALL_E experts): count per
// chunk of RS_CHUNK pairs, one CTA turns the counts into each chunk's first
// row per expert (and seg / active), then every chunk places its pairs with
// the same stable warp ranking as the one-CTA kernel. hist is
// [chunks][n_experts + 1] ints of caller scratch.
constexpr int RS_CHUNK = 4096;

__global__ void __launch_bounds__(RT_THREADS) route_count_kernel(const int64_t* __restrict__ topk, int T, int k, int E,
                                                                 int32_t* __restrict__ hist, int* err, int skip) {
  extern __shared__ int sm[];
  const int NB = E + 1, P = T * k;
  for (int b = threadIdx.x; b < NB; b += RT_THREADS) sm[b] = 0;
  __syncthreads();
  const int p0 = blockIdx.x * RS_CHUNK, p1 = min(P, p0 + RS_CHUNK);
  for (int p = p0 + threadIdx.x; p < p1; p += RT_THREADS) atomicAdd(&sm[pair_bucket(topk, T, k, E, p, err, skip)], 1);
  __syncthreads();
  for (int b = threadIdx.x; b < NB; b += RT_THREADS) hist[(int64_t)blockIdx.x * NB + b] = sm[b];
}

__global__ void __launch_bounds__(RT_THREADS) route_scan_kernel(int E, int n_chunks, int32_t* __restrict__ hist,
                                                                int32_t* __restrict__ seg, int32_t* __restrict__ active) {
  extern __shared__ int sm[];  // [NB] bucket totals
  const int NB = E + 1;
  for (int b = threadIdx.x; b < NB; b += RT_THREADS) {
    int t = 0;
    for (int c = 0; c < n_chunks; ++c) t += hist[(int64_t)c * NB + b];
    sm[b] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0, na = 0;
    for (int b = 0; b < NB; ++b) {
      const int c = sm[b];
      sm[b] = run;
      if (b < E) {
        seg[b] = run;
        if (c > 0) active[1 + na++] = b;
      }
      run += c;
    }
    seg[E] = sm[E];
    active[0] = na;
  }
  __syncthreads();
  for (int b = threadIdx.x; b < NB; b += RT_THREADS) {
    int run = sm[b];
    for (int c = 0; c < n_chunks; ++c) {
      const int h = hist[(int64_t)c * NB + b];
      hist[(int64_t)c * NB + b] = run;
      run += h;
    }
  }
}

__global__ void __launch_bounds__(RT_THREADS) route_scatter_kernel(const int64_t* __restrict__ topk, int T, int k,
                                                                   int E, const int32_t* __restrict__ hist,
                                                                   int32_t* __restrict__ perm,
                                                                   int32_t* __restrict__ inv, int* err, int skip) {
  extern __shared__ int sm[];
  const int NB = E + 1, P = T * k;
  int* base = sm;            // [NB]
  int* tot = base + NB;      // [NB]
  int* wcnt = tot + NB;      // [32][NB]
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  for (int b = tid; b < NB; b += RT_THREADS) base[b] = hist[(int64_t)blockIdx.x * NB + b];
  const int p0 = blockIdx.x * RS_CHUNK, p1 = min(P, p0 + RS_CHUNK);
  for (int c0 = p0; c0 < p1; c0 += RT_THREADS) {
    for (int i = tid; i < 32 * NB; i += RT_THREADS) wcnt[i] = 0;
    __syncthreads();
    const int p = c0 + tid;
    const int bk = p < p1 ? pair_bucket(topk, T, k, E, p, err, skip) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, bk);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (bk >= 0 && lane == __ffs(peers) - 1) wcnt[w * NB + bk] = __popc(peers);
    __syncthreads();
    for (int b = tid; b < NB; b += RT_THREADS) {
      int run = 0;
      for (int ww = 0; ww < 32; ++ww) {
        const int c = wcnt[ww * NB + b];
        wcnt[ww * NB + b] = run;
        run += c;
      }
      tot[b] = run;
    }
    __syncthreads();
    if (bk >= 0) {
      const int pos = base[bk] + wcnt[w * NB + bk] + rank;
      perm[pos] = p;
      inv[p] = pos;
    }
    __syncthreads();
    for (int b = tid; b < NB; b += RT_THREADS) base[b] += tot[b];
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Grouped codebook forward
// ---------------------------------------------------------------------------

constexpr int FW_THREADS = 128;  // outputs per CTA
constexpr int FW_ROWS = 8;       // most rows per shared-memory chunk (the kernel's R is 1, 2, 4 or 8)

// blocks whose centroid loads are issued together (more for small vectors)
template <int BS>
__host__ __device__ constexpr int fw_unroll() {
  return BS <= 4 ? 8 : (BS <= 8 ? 4 : 2);
}

struct FwdArgs {
  const void* x;
  int x_dtype;
  int64_t x_ld;
  const int32_t* row_token;  // row r reads x[row_token[r] % T] (NULL: x[r])
  int T;
  const int32_t* seg;
  const int32_t* seg_expert;
  const int32_t* active;
  int n_seg;
  int out_dim;
  int n_split;
  float* part;  // [n_split][P][out]
  int64_t P;
  int accumulate;
};

// acc[r] += scale * <xs[r][col0 + 0..BS), w> for the R rows of the chunk.
template <int BS, int R>
__device__ __forceinline__ void block_rows(const float* __restrict__ xs, int ld, int col0, const float (&w)[BS],
                                           bool scaled, float sc, float (&acc)[R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float d = 0.f;
#pragma unroll
    for (int j = 0; j < BS; ++j) d = __fmaf_rn(xs[r * ld + col0 + j], w[j], d);
    acc[r] = scaled ? __fmaf_rn(d, sc, acc[r]) : acc[r] + d;
  }
}

template <int BS, typename T, int R>
__device__ __forceinline__ void layer_rows(const skcq_fwd_layer& L, int e, int o, int out, int b0, int b1,
                                           const float* __restrict__ xs, int ld, bool last, float (&acc)[R]) {
  constexpr int FW_UNROLL = fw_unroll<BS>();
  const int nb = L.n_blocks;
  const T* table = static_cast<const T*>(L.table);
  const uint16_t* ix = L.idx16 + (int64_t)e * nb * out + o;
  const uint32_t* sg = L.sign_mask ? L.sign_mask + (int64_t)e * nb * out + o : nullptr;
  const bool scaled = L.scales != nullptr;
  int b = b0;
  for (; b + FW_UNROLL <= b1; b += FW_UNROLL) {
    int idx[FW_UNROLL];
#pragma unroll
    for (int u = 0; u < FW_UNROLL; ++u) idx[u] = __ldg(ix + (int64_t)(b + u) * out);
    float w[FW_UNROLL][BS];
#pragma unroll
    for (int u = 0; u < FW_UNROLL; ++u) load_centroid<BS, T>(table + ((int64_t)(b + u) * L.K + idx[u]) * BS, w[u]);
    float sc[FW_UNROLL];
    uint32_t m[FW_UNROLL];
#pragma unroll
    for (int u = 0; u < FW_UNROLL; ++u) {
      sc[u] = scaled ? ld_scale(L.scales, ((int64_t)e * nb + b + u) * out + o, L.scale_dtype, L.q_scale) : 1.f;
      m[u] = sg ? __ldg(sg + (int64_t)(b + u) * out) : 0u;
    }
#pragma unroll
    for (int u = 0; u < FW_UNROLL; ++u) {
#pragma unroll
      for (int j = 0; j < BS; ++j)
        if (m[u] >> j & 1u) w[u][j] = -w[u][j];
      block_rows<BS, R>(xs, ld, (b + u - b0) * BS, w[u], scaled, sc[u], acc);
    }
  }
  for (; b < b1; ++b) {
    const int idx = __ldg(ix + (int64_t)b * out);
    float w[BS];
    load_centroid<BS, T>(table + ((int64_t)b * L.K + idx) * BS, w);
    const float sc = scaled ? ld_scale(L.scales, ((int64_t)e * nb + b) * out + o, L.scale_dtype, L.q_scale) : 1.f;
    const uint32_t m = sg ? __ldg(sg + (int64_t)b * out) : 0u;
#pragma unroll
    for (int j = 0; j < BS; ++j)
      if (m >> j & 1u) w[j] = -w[j];
    block_rows<BS, R>(xs, ld, (b - b0) * BS, w, scaled, sc, acc);
  }
  if (last) {
    // raw remainder columns x[:, cov:cov+rem] @ rem_w[e].T (codebook_experts.py:64-74)
    const int c0 = (b1 - b0) * BS;
    for (int c = 0; c < L.rem; ++c) {
      const float wv = ld_any(L.remainder, ((int64_t)e * out + o) * L.rem + c, L.rem_dtype);
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = __fmaf_rn(xs[r * ld + c0 + c], wv, acc[r]);
    }
  }
}

// Generic block size (runtime bs <= 32): same arithmetic, scalar loads.
template <typename T, int R>
__device__ __forceinline__ void layer_rows_any(const skcq_fwd_layer& L, int e, int o, int out, int b0, int b1,
                                               const float* __restrict__ xs, int ld, bool last, float (&acc)[R]) {
  const int nb = L.n_blocks, bs = L.bs;
  const T* table = static_cast<const T*>(L.table);
  for (int b = b0; b < b1; ++b) {
    const int idx = L.idx16[((int64_t)e * nb + b) * out + o];
    const uint32_t m = L.sign_mask ? L.sign_mask[((int64_t)e * nb + b) * out + o] : 0u;
    const T* cp = table + ((int64_t)b * L.K + idx) * bs;
    float d[R];
#pragma unroll
    for (int r = 0; r < R; ++r) d[r] = 0.f;
    for (int j = 0; j < bs; ++j) {
      float w;
      if constexpr (sizeof(T) == 4)
        w = reinterpret_cast<const float*>(cp)[j];
      else
        w = __uint_as_float((uint32_t) reinterpret_cast<const uint16_t*>(cp)[j] << 16);
      if (m >> j & 1u) w = -w;
#pragma unroll
      for (int r = 0; r < R; ++r) d[r] = __fmaf_rn(xs[r * ld + (b - b0) * bs + j], w, d[r]);
    }
    if (L.scales) {
      const float sc = ld_scale(L.scales, ((int64_t)e * nb + b) * out + o, L.scale_dtype, L.q_scale);
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = __fmaf_rn(d[r], sc, acc[r]);
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] += d[r];
    }
  }
  if (last) {
    const int c0 = (b1 - b0) * bs;
    for (int c = 0; c < L.rem; ++c) {
      const float wv = ld_any(L.remainder, ((int64_t)e * out + o) * L.rem + c, L.rem_dtype);
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = __fmaf_rn(xs[r * ld + c0 + c], wv, acc[r]);
    }
  }
}

template <int BS, typename T, int R>
__device__ __forceinline__ void rows_dispatch(const skcq_fwd_layer& L, int e, int o, int out, int b0, int b1,
                                              const float* xs, int ld, bool last, float (&acc)[R]) {
  if constexpr (BS == 0)
    layer_rows_any<T, R>(L, e, o, out, b0, b1, xs, ld, last, acc);
  else
    layer_rows<BS, T, R>(L, e, o, out, b0, b1, xs, ld, last, acc);
}

// grid.x = n_split * (segments) * tiles, split slowest. BS == 0: runtime bs.
// R rows per shared-memory chunk: the host picks the smallest of 1, 2, 4, 8
// covering the expected rows per segment (decode: the batch size), so a
// single-token step runs a kernel with one accumulator per thread.
template <int BS, typename T, int R>
__global__ void __launch_bounds__(FW_THREADS) fwd_layer_kernel(FwdArgs a, skcq_fwd_layer L) {
  extern __shared__ float xs[];
  const int out = a.out_dim;
  const int tiles = (out + FW_THREADS - 1) / FW_THREADS;
  const int n_act = a.active ? a.active[0] : a.n_seg;
  const int per_split = n_act * tiles;
  const int item = blockIdx.x;
  if (item >= per_split * a.n_split) return;
  const int split = item / per_split;
  const int rest = item - split * per_split;
  const int ai = rest / tiles, tile = rest - ai * tiles;
  const int s = a.active ? a.active[1 + ai] : ai;
  const int r0 = a.seg[s], r1 = a.seg[s + 1];
  if (r0 >= r1) return;
  const int e = a.seg_expert ? a.seg_expert[s] : s;
  const int bs = BS == 0 ? L.bs : BS;
  const int nb = L.n_blocks;
  const int b0 = (int)((int64_t)nb * split / a.n_split), b1 = (int)((int64_t)nb * (split + 1) / a.n_split);
  const bool last = split == a.n_split - 1;
  const int nblk_cols = (b1 - b0) * bs;
  const int ncols = nblk_cols + (last ? L.rem : 0);
  const int cov = nb * bs;
  const int o = tile * FW_THREADS + threadIdx.x;
  const bool live = o < out;
  for (int rc = r0; rc < r1; rc += R) {
    const int nr = min(R, r1 - rc);
    __syncthreads();
    for (int i = threadIdx.x; i < R * ncols; i += FW_THREADS) {
      const int rr = i / ncols, c = i - rr * ncols;
      float v = 0.f;
      if (rr < nr) {
        const int col = c < nblk_cols ? b0 * bs + c : cov + (c - nblk_cols);
        const int row = rc + rr;
        const int64_t tok = a.row_token ? (int64_t)(a.row_token[row] % a.T) : (int64_t)row;
        v = ld_any(a.x, tok * a.x_ld + col, a.x_dtype);
      }
      xs[i] = v;
    }
    __syncthreads();
    if (!live) continue;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    rows_dispatch<BS, T, R>(L, e, o, out, b0, b1, xs, ncols, last, acc);
    float* dst = a.part + ((int64_t)split * a.P + rc) * out + o;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r < nr) {
        float v = acc[r];
        if (a.accumulate) v += dst[(int64_t)r * out];
        dst[(int64_t)r * out] = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Lookup-table decode (the reference's matmul_gather mode,
// codebook_experts.py:57-60): the per-token table of block dots is built once
// per layer and the forward reads one float per (row, block, output) instead
// of gathering a centroid vector. Each table entry is the block dot the gather
// kernel forms (same fused multiply-adds in the same order), so both paths
// produce identical bits.
// ---------------------------------------------------------------------------

constexpr int LUT_THREADS = 256;

// lut[(b K + k) T + t] = <x_b(t), C_b[k]>. One CTA per (block, 256 centroids);
// the block's columns of x are staged in shared memory, `chunk` rows at a time.
template <int BS, typename T>
__global__ void __launch_bounds__(LUT_THREADS) lut_build_kernel(skcq_fwd_layer L, const void* __restrict__ x,
                                                                int x_dtype, int64_t x_ld, int n_tok, int chunk,
                                                                float* __restrict__ lut) {
  extern __shared__ float xb[];  // [chunk][BS]
  const int b = blockIdx.y;
  const int k = blockIdx.x * LUT_THREADS + threadIdx.x;
  float w[BS];
  if (k < L.K) load_centroid<BS, T>(static_cast<const T*>(L.table) + ((int64_t)b * L.K + k) * BS, w);
  float* dst = lut + ((int64_t)b * L.K + k) * n_tok;
  for (int t0 = 0; t0 < n_tok; t0 += chunk) {
    const int nt = min(chunk, n_tok - t0);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * BS; i += LUT_THREADS) {
      const int t = i / BS, j = i - t * BS;
      xb[i] = ld_any(x, (int64_t)(t0 + t) * x_ld + (int64_t)b * BS + j, x_dtype);
    }
    __syncthreads();
    if (k >= L.K) continue;
    for (int t = 0; t < nt; ++t) {
      float d = 0.f;
#pragma unroll
      for (int j = 0; j < BS; ++j) d = __fmaf_rn(xb[t * BS + j], w[j], d);
      dst[t0 + t] = d;
    }
  }
}

// The forward of fwd_layer_kernel (same grid, rows, splits and partial sums)
// reading block dots from the layer's lookup table.
constexpr int LUT_UNROLL = 8;

template <int R>
__global__ void __launch_bounds__(FW_THREADS) fwd_lut_kernel(FwdArgs a, skcq_fwd_layer L) {
  extern __shared__ float xs[];  // [R][rem] remainder columns (last split)
  __shared__ int tok[R];
  const int out = a.out_dim;
  const int tiles = (out + FW_THREADS - 1) / FW_THREADS;
  const int n_act = a.active ? a.active[0] : a.n_seg;
  const int per_split = n_act * tiles;
  const int item = blockIdx.x;
  if (item >= per_split * a.n_split) return;
  const int split = item / per_split;
  const int rest = item - split * per_split;
  const int ai = rest / tiles, tile = rest - ai * tiles;
  const int s = a.active ? a.active[1 + ai] : ai;
  const int r0 = a.seg[s], r1 = a.seg[s + 1];
  if (r0 >= r1) return;
  const int e = a.seg_expert ? a.seg_expert[s] : s;
  const int nb = L.n_blocks;
  const int b0 = (int)((int64_t)nb * split / a.n_split), b1 = (int)((int64_t)nb * (split + 1) / a.n_split);
  const bool last = split == a.n_split - 1;
  const int cov = nb * L.bs;
  const int rem = last ? L.rem : 0;
  const int o = tile * FW_THREADS + threadIdx.x;
  const bool live = o < out;
  const int64_t K = L.K;
  const int nt = L.lut_tokens;
  for (int rc = r0; rc < r1; rc += R) {
    const int nr = min(R, r1 - rc);
    __syncthreads();
    if (threadIdx.x < R) {
      const int row = rc + min((int)threadIdx.x, nr - 1);
      tok[threadIdx.x] = a.row_token ? (int)(a.row_token[row] % a.T) : row;
    }
    for (int i = threadIdx.x; i < R * rem; i += FW_THREADS) {
      const int rr = i / rem, c = i - rr * rem;
      float v = 0.f;
      if (rr < nr) {
        const int row = rc + rr;
        const int64_t tk = a.row_token ? (int64_t)(a.row_token[row] % a.T) : (int64_t)row;
        v = ld_any(a.x, tk * a.x_ld + cov + c, a.x_dtype);
      }
      xs[i] = v;
    }
    __syncthreads();
    if (!live) continue;
    int tr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) tr[r] = tok[r];
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    const uint16_t* ix = L.idx16 + (int64_t)e * nb * out + o;
    const bool scaled = L.scales != nullptr;
    int b = b0;
    for (; b + LUT_UNROLL <= b1; b += LUT_UNROLL) {
      int idx[LUT_UNROLL];
#pragma unroll
      for (int u = 0; u < LUT_UNROLL; ++u) idx[u] = __ldg(ix + (int64_t)(b + u) * out);
      float d[LUT_UNROLL][R];
#pragma unroll
      for (int u = 0; u < LUT_UNROLL; ++u) {
        const float* base = L.lut + ((int64_t)(b + u) * K + idx[u]) * nt;
#pragma unroll
        for (int r = 0; r < R; ++r) d[u][r] = __ldg(base + tr[r]);
      }
#pragma unroll
      for (int u = 0; u < LUT_UNROLL; ++u) {
        const float sc =
            scaled ? ld_scale(L.scales, ((int64_t)e * nb + b + u) * out + o, L.scale_dtype, L.q_scale) : 1.f;
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] = scaled ? __fmaf_rn(d[u][r], sc, acc[r]) : acc[r] + d[u][r];
      }
    }
    for (; b < b1; ++b) {
      const int idx = __ldg(ix + (int64_t)b * out);
      const float* base = L.lut + ((int64_t)b * K + idx) * nt;
      const float sc = scaled ? ld_scale(L.scales, ((int64_t)e * nb + b) * out + o, L.scale_dtype, L.q_scale) : 1.f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float d = __ldg(base + tr[r]);
        acc[r] = scaled ? __fmaf_rn(d, sc, acc[r]) : acc[r] + d;
      }
    }
    // raw remainder columns x[:, cov:cov+rem] @ rem_w[e].T (codebook_experts.py:64-74)
    for (int c = 0; c < rem; ++c) {
      const float wv = ld_any(L.remainder, ((int64_t)e * out + o) * L.rem + c, L.rem_dtype);
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = __fmaf_rn(xs[r * rem + c], wv, acc[r]);
    }
    float* dst = a.part + ((int64_t)split * a.P + rc) * out + o;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r < nr) {
        float v = acc[r];
        if (a.accumulate) v += dst[(int64_t)r * out];
        dst[(int64_t)r * out] = v;
      }
    }
  }
}

static void launch_lut(const FwdArgs& a, const skcq_fwd_layer& L, int R, int grid, cudaStream_t s) {
  const size_t smem = (size_t)R * L.rem * sizeof(float);
  switch (R) {
    case 1: fwd_lut_kernel<1><<<grid, FW_THREADS, smem, s>>>(a, L); break;
    case 2: fwd_lut_kernel<2><<<grid, FW_THREADS, smem, s>>>(a, L); break;
    case 4: fwd_lut_kernel<4><<<grid, FW_THREADS, smem, s>>>(a, L); break;
    default: fwd_lut_kernel<8><<<grid, FW_THREADS, smem, s>>>(a, L); break;
  }
}

template <int BS, int R>
void launch_layer_r(const FwdArgs& a, const skcq_fwd_layer& L, int grid, size_t smem, cudaStream_t s) {
  if (L.table_dtype == SKCQ_DTYPE_BF16)
    fwd_layer_kernel<BS, __nv_bfloat16, R><<<grid, FW_THREADS, smem, s>>>(a, L);
  else
    fwd_layer_kernel<BS, float, R><<<grid, FW_THREADS, smem, s>>>(a, L);
}

template <int BS>
void launch_layer(const FwdArgs& a, const skcq_fwd_layer& L, int R, int grid, size_t smem, cudaStream_t s) {
  switch (R) {
    case 1: launch_layer_r<BS, 1>(a, L, grid, smem, s); break;
    case 2: launch_layer_r<BS, 2>(a, L, grid, smem, s); break;
    case 4: launch_layer_r<BS, 4>(a, L, grid, smem, s); break;
    default: launch_layer_r<BS, 8>(a, L, grid, smem, s); break;
  }
}

template <int BS, int R>
cudaError_t allow_smem_r() {
  cudaError_t e = cudaFuncSetAttribute(fwd_layer_kernel<BS, __nv_bfloat16, R>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(fwd_layer_kernel<BS, float, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  return e;
}

template <int BS>
cudaError_t allow_smem() {
  cudaError_t e = allow_smem_r<BS, 1>();
  if (e == cudaSuccess) e = allow_smem_r<BS, 2>();
  if (e == cudaSuccess) e = allow_smem_r<BS, 4>();
  if (e == cudaSuccess) e = allow_smem_r<BS, 8>();
  return e;
}

// ---------------------------------------------------------------------------
// Consumers of the split partial sums
// ---------------------------------------------------------------------------

__device__ __forceinline__ float sum_parts(const float* __restrict__ part, int n_split, int64_t stride, int64_t i) {
  float v = part[i];
  for (int s = 1; s < n_split; ++s) v += part[s * stride + i];
  return v;
}

// y[r][o] = sum_s part[s][r][o]
__global__ void sum_splits_kernel(const float* __restrict__ part, int n_split, int64_t P, int out, void* __restrict__ y,
                                  int y_dtype, int64_t y_ld) {
  const int64_t total = P * out;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / out, o = i - r * out;
    st_any(y, r * y_ld + o, y_dtype, sum_parts(part, n_split, total, i));
  }
}

// inter = silu(gate) * up (the _SwiGLU of codebook_experts.py:427-433 with act = SiLU)
__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, int n_split, int64_t n,
                              float* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float a = sum_parts(g, n_split, n, i);
    out[i] = __fdiv_rn(a, 1.0f + expf(-a)) * sum_parts(u, n_split, n, i);
  }
}

// out[t][h] = sum over the token's k slots, in ascending (expert, kpos) order,
// of y(pair) * w[t][kpos] (codebook_experts.py:476-480: multiply, then index_add_).
// A CTA owns one token and a stripe of h (grid.y stripes, so a one-token
// decode step still spreads over the SMs): the slot order is resolved once in
// shared memory, then the threads stream the token's k rows over h.
constexpr int CB_THREADS = 256;

__global__ void __launch_bounds__(CB_THREADS) combine_kernel(const void* __restrict__ part, int part_dtype,
                                                             int n_split, int64_t P,
                                                             const int32_t* __restrict__ row_of_pair,
                                                             const int64_t* __restrict__ topk, const void* __restrict__ w,
                                                             int w_dtype, int T, int k, int H, void* __restrict__ out,
                                                             int out_dtype, int vec8) {
  __shared__ int s_row[32];
  __shared__ float s_w[32];
  __shared__ int s_n;
  const int64_t stride = P * H;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    if (threadIdx.x < 32) {
      // lane kp ranks its slot by (expert, kpos) among the token's k slots
      // (a negative id: a slot routed elsewhere, skipped)
      const int lane = threadIdx.x;
      int64_t e = lane < k ? topk[(int64_t)t * k + lane] : INT64_MAX;
      if (e < 0) e = INT64_MAX;
      int rank = 0;
      for (int j = 0; j < k; ++j) {
        const int64_t ej = __shfl_sync(0xffffffffu, e, j);
        rank += (ej < e || (ej == e && j < lane)) ? 1 : 0;
      }
      const unsigned live = __ballot_sync(0xffffffffu, lane < k && e != INT64_MAX);
      if (lane == 0) s_n = __popc(live);
      if (lane < k) {
        s_row[rank] = row_of_pair[(int64_t)lane * T + t];
        s_w[rank] = ld_any(w, (int64_t)t * k + lane, w_dtype);
      }
    }
    __syncthreads();
    const int n_live = s_n;
    if (vec8) {
      // bf16 pair outputs, one split, H % 8 == 0: 16-byte loads and stores of
      // 8 consecutive features, the same arithmetic per feature
      for (int h = (blockIdx.y * CB_THREADS + threadIdx.x) * 8; h < H; h += gridDim.y * CB_THREADS * 8) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int step = 0; step < n_live; ++step) {
          float y[8];
          ld_bf16x8(part, (int64_t)s_row[step] * H + h, y);
          const float ws = s_w[step];
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(y[j], ws));
        }
        st_x8(out, (int64_t)t * H + h, out_dtype, acc);
      }
    } else {
      for (int h = blockIdx.y * CB_THREADS + threadIdx.x; h < H; h += gridDim.y * CB_THREADS) {
        float acc = 0.f;
        for (int step = 0; step < n_live; ++step) {
          const int64_t i = (int64_t)s_row[step] * H + h;
          float y = ld_any(part, i, part_dtype);
          for (int sp = 1; sp < n_split; ++sp) y += ld_any(part, sp * stride + i, part_dtype);
          acc = __fadd_rn(acc, __fmul_rn(y, s_w[step]));
        }
        st_any(out, (int64_t)t * H + h, out_dtype, acc);
      }
    }
    __syncthreads();
  }
}

}  // namespace skcq

using namespace skcq;

extern "C" int skcq_pack_indices16(const int64_t* idx, int64_t n, int K, uint16_t* out, void* stream) {
  SKCQ_REQUIRE(idx && out, SKCQ_ERR_INVALID, "pack_indices16: null pointer");
  SKCQ_REQUIRE(K > 0 && K <= 65536, SKCQ_ERR_INVALID, "pack_indices16: codebook size %d outside [1, 65536]", K);
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "pack_indices16: no device error word");
  if (n <= 0) return SKCQ_OK;
  pack_idx16_kernel<<<gridf(n), 256, 0, (cudaStream_t)stream>>>(idx, n, K, out, err);
  return check_launch("pack_indices16");
}

extern "C" int skcq_transpose_codebook(const void* cb, int dtype, int n_blocks, int bs, int K, void* table,
                                       void* stream) {
  SKCQ_REQUIRE(cb && table, SKCQ_ERR_INVALID, "transpose_codebook: null pointer");
  SKCQ_REQUIRE(dtype == SKCQ_DTYPE_F32 || dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "transpose_codebook: dtype %d is not f32 or bf16", dtype);
  SKCQ_REQUIRE(n_blocks >= 0 && bs > 0 && K > 0, SKCQ_ERR_INVALID, "transpose_codebook: bad sizes");
  const int64_t total = (int64_t)n_blocks * K;
  if (total == 0) return SKCQ_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (dtype == SKCQ_DTYPE_BF16)
    transpose_cb_kernel<uint16_t><<<gridf(total), 256, 0, s>>>(static_cast<const uint16_t*>(cb), n_blocks, bs, K,
                                                              static_cast<uint16_t*>(table));
  else
    transpose_cb_kernel<float><<<gridf(total), 256, 0, s>>>(static_cast<const float*>(cb), n_blocks, bs, K,
                                                           static_cast<float*>(table));
  return check_launch("transpose_codebook");
}

extern "C" int skcq_pack_sign_masks(const int8_t* signs, int E, int out, int64_t sign_ld, int n_blocks, int bs,
                                    uint32_t* mask, void* stream) {
  SKCQ_REQUIRE(signs && mask, SKCQ_ERR_INVALID, "pack_sign_masks: null pointer");
  SKCQ_REQUIRE(bs > 0 && bs <= 32, SKCQ_ERR_INVALID, "pack_sign_masks: block size %d outside [1, 32]", bs);
  SKCQ_REQUIRE(sign_ld >= (int64_t)n_blocks * bs, SKCQ_ERR_INVALID,
               "pack_sign_masks: signs cover %lld columns, blocks need %lld", (long long)sign_ld,
               (long long)n_blocks * bs);
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "pack_sign_masks: no device error word");
  const int64_t total = (int64_t)E * n_blocks * out;
  if (total <= 0) return SKCQ_OK;
  pack_signs_kernel<<<gridf(total), 256, 0, (cudaStream_t)stream>>>(signs, E, out, sign_ld, n_blocks, bs, mask, err);
  return check_launch("pack_sign_masks");
}

extern "C" size_t skcq_route_sort_scratch_bytes(int T, int k, int n_experts) {
  const int64_t P = (int64_t)T * k;
  if (T <= 0 || k <= 0 || n_experts <= 0 || n_experts > RT_SMALL_E || P <= RS_CHUNK) return 0;
  return (size_t)((P + RS_CHUNK - 1) / RS_CHUNK) * (size_t)(n_experts + 1) * sizeof(int32_t);
}

extern "C" int skcq_route_sort(const int64_t* topk, int T, int k, int n_experts, int32_t* perm, int32_t* seg,
                               int32_t* row_of_pair, int32_t* active, void* scratch, size_t scratch_bytes,
                               int skip_negative, void* stream) {
  SKCQ_REQUIRE(topk && perm && seg && row_of_pair && active, SKCQ_ERR_INVALID, "route_sort: null pointer");
  SKCQ_REQUIRE(T >= 0 && k > 0 && k <= 31 && n_experts > 0 && n_experts <= 8192, SKCQ_ERR_INVALID,
               "route_sort: bad sizes (T %d, k %d, experts %d)", T, k, n_experts);
  SKCQ_REQUIRE((int64_t)T * k < (1LL << 31), SKCQ_ERR_INVALID, "route_sort: %lld pairs", (long long)T * k);
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "route_sort: no device error word");
  const int NB = n_experts + 1;
  const size_t need = skcq_route_sort_scratch_bytes(T, k, n_experts);
  if (need > 0 && scratch != nullptr && scratch_bytes >= need) {
    cudaStream_t s = (cudaStream_t)stream;
    const int P = T * k;
    const int chunks = (P + RS_CHUNK - 1) / RS_CHUNK;
    int32_t* hist = static_cast<int32_t*>(scratch);
    route_count_kernel<<<chunks, RT_THREADS, (size_t)NB * sizeof(int), s>>>(topk, T, k, n_experts, hist, err,
                                                                            skip_negative);
    route_scan_kernel<<<1, RT_THREADS, (size_t)NB * sizeof(int), s>>>(n_experts, chunks, hist, seg, active);
    route_scatter_kernel<<<chunks, RT_THREADS, (size_t)34 * NB * sizeof(int), s>>>(topk, T, k, n_experts, hist, perm,
                                                                                   row_of_pair, err, skip_negative);
    return check_launch("route_sort");
  }
  size_t smem = (size_t)3 * NB * sizeof(int);
  if (n_experts <= RT_SMALL_E) smem += (size_t)32 * NB * sizeof(int);
  route_sort_kernel<<<1, RT_THREADS, smem, (cudaStream_t)stream>>>(topk, T, k, n_experts, perm, seg, row_of_pair,
                                                                  active, err, skip_negative);
  return check_launch("route_sort");
}

extern "C" int skcq_codebook_forward(const skcq_fwd_layer* layers, int n_layers, const void* x, int x_dtype,
                                     int64_t x_ld, const int32_t* row_token, int T, const int32_t* seg,
                                     const int32_t* seg_expert, const int32_t* active, int n_seg, int max_active,
                                     int in_dim, int out_dim, int n_split, int rows_hint, float* part, int64_t P,
                                     void* stream) {
  SKCQ_REQUIRE(layers && x && seg && part, SKCQ_ERR_INVALID, "codebook_forward: null pointer");
  SKCQ_REQUIRE(x_dtype == SKCQ_DTYPE_F32 || x_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "codebook_forward: x dtype %d", x_dtype);
  SKCQ_REQUIRE(n_layers >= 1 && n_layers <= SKCQ_MAX_CODECS, SKCQ_ERR_INVALID, "codebook_forward: %d layers",
               n_layers);
  SKCQ_REQUIRE(n_seg >= 0 && max_active >= 0 && max_active <= n_seg, SKCQ_ERR_INVALID,
               "codebook_forward: %d segments, %d active", n_seg, max_active);
  SKCQ_REQUIRE(n_split >= 1 && n_split <= 256, SKCQ_ERR_INVALID, "codebook_forward: %d splits", n_split);
  SKCQ_REQUIRE(row_token == nullptr || T > 0, SKCQ_ERR_INVALID, "codebook_forward: token map without tokens");
  const int R = rows_hint <= 1 ? 1 : rows_hint <= 2 ? 2 : rows_hint <= 4 ? 4 : FW_ROWS;
  size_t smem_max = 0;
  for (int i = 0; i < n_layers; ++i) {
    const skcq_fwd_layer& L = layers[i];
    SKCQ_REQUIRE(L.table && L.idx16 && L.bs > 0 && L.bs <= 32 && L.n_blocks >= 0 && L.K > 0 && L.K <= 65536,
                 SKCQ_ERR_INVALID, "codebook_forward: layer %d incomplete or bs %d / K %d out of range", i, L.bs,
                 L.K);
    SKCQ_REQUIRE(L.table_dtype == SKCQ_DTYPE_F32 || L.table_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
                 "codebook_forward: layer %d table dtype %d", i, L.table_dtype);
    SKCQ_REQUIRE(L.n_blocks * L.bs + L.rem <= in_dim, SKCQ_ERR_INVALID,
                 "codebook_forward: layer %d covers %d columns of %d", i, L.n_blocks * L.bs + L.rem, in_dim);
    SKCQ_REQUIRE(L.rem == 0 || L.remainder, SKCQ_ERR_INVALID, "codebook_forward: layer %d remainder missing", i);
    SKCQ_REQUIRE(L.rem == 0 || L.rem_dtype == SKCQ_DTYPE_F32 || L.rem_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
                 "codebook_forward: layer %d remainder dtype %d", i, L.rem_dtype);
    if (L.lut) {
      SKCQ_REQUIRE(L.sign_mask == nullptr, SKCQ_ERR_INVALID,
                   "codebook_forward: layer %d has signs; its lookup table cannot apply them", i);
      SKCQ_REQUIRE(row_token ? L.lut_tokens == T : L.lut_tokens >= P, SKCQ_ERR_INVALID,
                   "codebook_forward: layer %d lookup table covers %d rows of x (need %lld)", i, L.lut_tokens,
                   row_token ? (long long)T : (long long)P);
      SKCQ_REQUIRE((size_t)R * L.rem * sizeof(float) <= 48 * 1024, SKCQ_ERR_INVALID,
                   "codebook_forward: layer %d remainder of %d columns too wide for the lookup path", i, L.rem);
      continue;
    }
    const int per = (L.n_blocks + n_split - 1) / n_split;
    const size_t smem = (size_t)R * (per * L.bs + L.rem) * sizeof(float);
    if (smem > smem_max) smem_max = smem;
  }
  SKCQ_REQUIRE(smem_max <= 200 * 1024, SKCQ_ERR_INVALID, "codebook_forward: %zu bytes of rows per CTA", smem_max);
  const int tiles = ceil_div(out_dim, FW_THREADS);
  const int64_t grid64 = (int64_t)n_split * max_active * tiles;
  if (grid64 == 0 || out_dim <= 0) return SKCQ_OK;
  SKCQ_REQUIRE(grid64 < (1LL << 31), SKCQ_ERR_INVALID, "codebook_forward: grid too large");
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaError_t e = allow_smem<0>();
    if (e == cudaSuccess) e = allow_smem<4>();
    if (e == cudaSuccess) e = allow_smem<6>();
    if (e == cudaSuccess) e = allow_smem<8>();
    if (e == cudaSuccess) e = allow_smem<12>();
    if (e == cudaSuccess) e = allow_smem<16>();
    if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "codebook_forward: %s", cudaGetErrorString(e));
    configured_dev = dev;
  }
  cudaStream_t s = (cudaStream_t)stream;
  FwdArgs a{x, x_dtype, x_ld, row_token, T, seg, seg_expert, active, n_seg, out_dim, n_split, part, P, 0};
  for (int i = 0; i < n_layers; ++i) {
    const skcq_fwd_layer& L = layers[i];
    const int per = (L.n_blocks + n_split - 1) / n_split;
    const size_t smem = (size_t)R * (per * L.bs + L.rem) * sizeof(float);
    a.accumulate = i > 0;
    if (L.lut) {
      launch_lut(a, L, R, (int)grid64, s);
      int rc = check_launch("codebook_forward (lookup table)");
      if (rc != SKCQ_OK) return rc;
      continue;
    }
    switch (L.bs) {
      case 4: launch_layer<4>(a, L, R, (int)grid64, smem, s); break;
      case 6: launch_layer<6>(a, L, R, (int)grid64, smem, s); break;
      case 8: launch_layer<8>(a, L, R, (int)grid64, smem, s); break;
      case 12: launch_layer<12>(a, L, R, (int)grid64, smem, s); break;
      case 16: launch_layer<16>(a, L, R, (int)grid64, smem, s); break;
      default: launch_layer<0>(a, L, R, (int)grid64, smem, s); break;
    }
    int rc = check_launch("codebook_forward");
    if (rc != SKCQ_OK) return rc;
  }
  return SKCQ_OK;
}

extern "C" int skcq_lut_build(const skcq_fwd_layer* layer, const void* x, int x_dtype, int64_t x_ld, int T, float* lut,
                              void* stream) {
  SKCQ_REQUIRE(layer && x && lut, SKCQ_ERR_INVALID, "lut_build: null pointer");
  const skcq_fwd_layer& L = *layer;
  SKCQ_REQUIRE(L.table && L.bs > 0 && L.bs <= 32 && L.K > 0 && L.n_blocks >= 0, SKCQ_ERR_INVALID,
               "lut_build: layer incomplete or bs %d / K %d out of range", L.bs, L.K);
  SKCQ_REQUIRE(L.table_dtype == SKCQ_DTYPE_F32 || L.table_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "lut_build: table dtype %d", L.table_dtype);
  SKCQ_REQUIRE(x_dtype == SKCQ_DTYPE_F32 || x_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID, "lut_build: x dtype %d",
               x_dtype);
  SKCQ_REQUIRE(T >= 1, SKCQ_ERR_INVALID, "lut_build: %d rows", T);
  const int chunk = T < 1024 ? T : 1024;  // rows staged at a time (<= 128 KB at bs 32)
  const size_t smem = (size_t)chunk * L.bs * sizeof(float);
  SKCQ_REQUIRE(L.n_blocks <= 65535, SKCQ_ERR_INVALID, "lut_build: %d blocks", L.n_blocks);
  if (L.n_blocks == 0) return SKCQ_OK;
  const dim3 grid((unsigned)ceil_div(L.K, LUT_THREADS), (unsigned)L.n_blocks);
  cudaStream_t s = (cudaStream_t)stream;
  const bool bf = L.table_dtype == SKCQ_DTYPE_BF16;
#define SKCQ_LUT_CASE(BSV)                                                                                   \
  case BSV:                                                                                                  \
    if (bf) {                                                                                                \
      cudaFuncSetAttribute(lut_build_kernel<BSV, __nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           160 * 1024);                                                                      \
      lut_build_kernel<BSV, __nv_bfloat16><<<grid, LUT_THREADS, smem, s>>>(L, x, x_dtype, x_ld, T, chunk, lut); \
    } else {                                                                                                 \
      cudaFuncSetAttribute(lut_build_kernel<BSV, float>, cudaFuncAttributeMaxDynamicSharedMemorySize,         \
                           160 * 1024);                                                                      \
      lut_build_kernel<BSV, float><<<grid, LUT_THREADS, smem, s>>>(L, x, x_dtype, x_ld, T, chunk, lut);      \
    }                                                                                                        \
    break;
  switch (L.bs) {
    SKCQ_LUT_CASE(4)
    SKCQ_LUT_CASE(6)
    SKCQ_LUT_CASE(8)
    SKCQ_LUT_CASE(12)
    SKCQ_LUT_CASE(16)
    default:
      return set_error(SKCQ_ERR_INVALID, "lut_build: block size %d has no lookup-table kernel (4, 6, 8, 12, 16)",
                       L.bs);
  }
#undef SKCQ_LUT_CASE
  return check_launch("lut_build");
}

extern "C" int skcq_sum_splits(const float* part, int n_split, int64_t P, int out_dim, void* y, int y_dtype,
                               int64_t y_ld, void* stream) {
  SKCQ_REQUIRE(part && y, SKCQ_ERR_INVALID, "sum_splits: null pointer");
  SKCQ_REQUIRE(n_split >= 1 && (y_dtype == SKCQ_DTYPE_F32 || y_dtype == SKCQ_DTYPE_BF16), SKCQ_ERR_INVALID,
               "sum_splits: %d splits, dtype %d", n_split, y_dtype);
  if (P * out_dim <= 0) return SKCQ_OK;
  sum_splits_kernel<<<gridf(P * out_dim), 256, 0, (cudaStream_t)stream>>>(part, n_split, P, out_dim, y, y_dtype,
                                                                          y_ld);
  return check_launch("sum_splits");
}

extern "C" int skcq_swiglu(const float* gate, const float* up, int n_split, int64_t n, float* out, void* stream) {
  SKCQ_REQUIRE(gate && up && out, SKCQ_ERR_INVALID, "swiglu: null pointer");
  SKCQ_REQUIRE(n_split >= 1, SKCQ_ERR_INVALID, "swiglu: %d splits", n_split);
  if (n <= 0) return SKCQ_OK;
  swiglu_kernel<<<gridf(n), 256, 0, (cudaStream_t)stream>>>(gate, up, n_split, n, out);
  return check_launch("swiglu");
}

extern "C" int skcq_combine(const void* part, int part_dtype, int n_split, int64_t P, const int32_t* row_of_pair,
                            const int64_t* topk, const void* weights, int w_dtype, int T, int k, int H, void* out,
                            int out_dtype, void* stream) {
  SKCQ_REQUIRE(part && row_of_pair && topk && weights && out, SKCQ_ERR_INVALID, "combine: null pointer");
  SKCQ_REQUIRE(part_dtype == SKCQ_DTYPE_F32 || part_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "combine: partial-sum dtype %d", part_dtype);
  SKCQ_REQUIRE(k > 0 && k <= 31 && n_split >= 1, SKCQ_ERR_INVALID, "combine: top-k %d, %d splits", k, n_split);
  SKCQ_REQUIRE(w_dtype == SKCQ_DTYPE_F32 || w_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID, "combine: weight dtype %d",
               w_dtype);
  SKCQ_REQUIRE(out_dtype == SKCQ_DTYPE_F32 || out_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "combine: output dtype %d", out_dtype);
  if ((int64_t)T * H <= 0) return SKCQ_OK;
  const int vec8 = part_dtype == SKCQ_DTYPE_BF16 && n_split == 1 && H % 8 == 0 && ((uintptr_t)part & 15) == 0 &&
                   ((uintptr_t)out & 15) == 0;
  const int gx = T < 148 * 16 ? T : 148 * 16;
  int gy = ceil_div(vec8 ? H / 8 : H, CB_THREADS);
  const int want_y = ceil_div(148 * 4, gx);
  if (gy > want_y) gy = want_y;
  combine_kernel<<<dim3(gx, gy), CB_THREADS, 0, (cudaStream_t)stream>>>(part, part_dtype, n_split, P, row_of_pair,
                                                                        topk, weights, w_dtype, T, k, H, out,
                                                                        out_dtype, vec8);
  return check_launch("combine");
}
