// Lloyd update, empty-cluster reseed and finalisation for the batched k-means
// problem sets (skcq/codebook/kmeans.py:152-188 cosine, 210-244 euclidean).
#include <mutex>

#include "common.cuh"

namespace skcq {

// ---------------------------------------------------------------------------
// Update: segmented sums + counts
// ---------------------------------------------------------------------------

// Shared-memory accumulation: one CTA owns a slice of rows of one problem and
// the whole (k x (bs+1)) accumulator; flushed with one global atomic per
// touched entry.
// Per-CTA partial sums in shared memory, flushed to global with atomics.
// blockIdx.z selects a pass over columns [j0, j0 + jn) of the points (several
// passes when a cluster row of all bs sums does not fit); pass 0 also counts.
// Cluster c's row is acc[c * sp .. c * sp + jn) with its count (as int) in
// column jn; the row stride sp = (jn + 1) | 1 is odd, so the 32 random clusters
// a warp touches spread over the banks instead of landing on the few banks a
// stride that is a multiple of 4 or 8 maps them to. Each thread loads the
// labels and coordinates of UP points before issuing their atomics, to keep
// several global loads in flight.
constexpr int UP = 4;
constexpr int UPDATE_SMEM = 160 * 1024;

__host__ __device__ constexpr int update_row_stride(int jn) { return (jn + 1) | 1; }

__global__ void __launch_bounds__(512) update_smem_kernel(const float* __restrict__ R,
                                                          const int32_t* __restrict__ labels, int n_pad, int k_pad,
                                                          int bs, int cols_per_pass, const int32_t* __restrict__ n,
                                                          const int32_t* __restrict__ active,
                                                          const int32_t* __restrict__ kvec, int rows_per_cta,
                                                          float* __restrict__ sums, int32_t* __restrict__ counts,
                                                          const uint8_t* __restrict__ changed) {
  extern __shared__ float acc[];  // [kb][sp]: jn sums, then the count (as int)
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int nb = n[b], kb = kvec[b];
  const int i0 = blockIdx.x * rows_per_cta;
  if (i0 >= nb) return;
  const int i1 = min(nb, i0 + rows_per_cta);
  const int j0 = blockIdx.z * cols_per_pass;
  const int jn = min(cols_per_pass, bs - j0);
  const bool counting = blockIdx.z == 0;
  const int sp = update_row_stride(jn);
  for (int t = threadIdx.x; t < kb * sp; t += blockDim.x) acc[t] = 0.f;
  __syncthreads();
  const float* Rb = R + (int64_t)b * n_pad * bs + j0;
  const int32_t* Lb = labels + (int64_t)b * n_pad;
  // rows are 16-byte aligned: R is [nblk][n_pad][bs] from an aligned base
  const bool vec4 = (bs & 3) == 0 && (j0 & 3) == 0 && (jn & 3) == 0;
  const uint8_t* Chb = changed ? changed + (int64_t)b * k_pad : nullptr;
  for (int base = i0 + threadIdx.x; base < i1; base += UP * blockDim.x) {
    int l[UP];
    bool sum_it[UP];  // false: the cluster kept its members, its centroid is kept (count only)
#pragma unroll
    for (int u = 0; u < UP; ++u) {
      const int i = base + u * blockDim.x;
      const int v = i < i1 ? Lb[i] : -1;
      l[u] = v < kb ? v : -1;  // a label outside [0, k) never indexes the accumulator
      sum_it[u] = l[u] >= 0 && (!Chb || Chb[l[u]]);
    }
    if (jn <= 16) {
      float x[UP][16];
#pragma unroll
      for (int u = 0; u < UP; ++u) {
        if (!sum_it[u]) continue;
        const float* xr = Rb + (int64_t)(base + u * blockDim.x) * bs;
        if (vec4) {
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            if (j < jn) {
              const float4 q = __ldg(reinterpret_cast<const float4*>(xr + j));
              x[u][j] = q.x; x[u][j + 1] = q.y; x[u][j + 2] = q.z; x[u][j + 3] = q.w;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < jn) x[u][j] = __ldg(xr + j);
        }
      }
#pragma unroll
      for (int u = 0; u < UP; ++u) {
        if (l[u] < 0) continue;
        float* row = acc + (size_t)l[u] * sp;
        if (sum_it[u]) {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (j < jn) atomicAdd(row + j, x[u][j]);
        }
        if (counting) atomicAdd(reinterpret_cast<int*>(row + jn), 1);
      }
    } else {
#pragma unroll
      for (int u = 0; u < UP; ++u) {
        if (l[u] < 0) continue;
        const float* xr = Rb + (int64_t)(base + u * blockDim.x) * bs;
        float* row = acc + (size_t)l[u] * sp;
        if (sum_it[u])
          for (int j = 0; j < jn; ++j) atomicAdd(row + j, xr[j]);
        if (counting) atomicAdd(reinterpret_cast<int*>(row + jn), 1);
      }
    }
  }
  __syncthreads();
  float* Sb = sums + (int64_t)b * k_pad * bs + j0;
  int32_t* Cb = counts + (int64_t)b * k_pad;
  for (int c = threadIdx.x; c < kb; c += blockDim.x) {
    const float* row = acc + (size_t)c * sp;
    if (counting) {
      const int m = __float_as_int(row[jn]);
      if (m == 0) continue;
      atomicAdd(&Cb[c], m);
    }
    for (int j = 0; j < jn; ++j) {
      const float v = row[j];
      if (v != 0.f || counting) atomicAdd(&Sb[(int64_t)c * bs + j], v);
    }
  }
}

__global__ void update_global_kernel(const float* __restrict__ R, const int32_t* __restrict__ labels, int nblk,
                                     int n_pad, int k_pad, int bs, const int32_t* __restrict__ n,
                                     const int32_t* __restrict__ active, float* __restrict__ sums,
                                     int32_t* __restrict__ counts, const uint8_t* __restrict__ changed) {
  const int64_t total = (int64_t)nblk * n_pad;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = t / n_pad, i = t % n_pad;
    if (i >= n[b] || (active && !active[b])) continue;
    const int l = labels[t];
    if (!changed || changed[b * k_pad + l]) {  // else the cluster kept its members: count only
      const float* x = R + t * bs;
      float* s = sums + (b * k_pad + l) * bs;
      for (int j = 0; j < bs; ++j) atomicAdd(&s[j], x[j]);
    }
    atomicAdd(&counts[b * k_pad + l], 1);
  }
}

// ---------------------------------------------------------------------------
// Reseed: worst-fit points into empty clusters
// ---------------------------------------------------------------------------

constexpr int RS_THREADS = 1024;
constexpr int RS_SMEM_SORT = 4096;  // sort in shared memory up to this many keys

__device__ __forceinline__ uint64_t reseed_key(int metric, const float* x, const float* c, int bs, int i) {
  uint32_t k;
  if (metric == SKCQ_METRIC_COSINE) {
    // kmeans.py:169-171: sims = <unit_x, c_label>, ascending
    float s = 0.f;
    for (int j = 0; j < bs; ++j) s = __fmaf_rn(x[j], c[j], s);
    k = float_key(s);
  } else {
    // kmeans.py:227-229: dists = ||x - c_label||^2, descending
    float s = 0.f;
    for (int j = 0; j < bs; ++j) {
      const float d = __fsub_rn(x[j], c[j]);
      s = __fmaf_rn(d, d, s);
    }
    k = ~float_key(s);
  }
  return ((uint64_t)k << 32) | (uint32_t)i;
}

__device__ void bitonic_sort(uint64_t* a, int P) {
  for (int k = 2; k <= P; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < P; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t x = a[i], y = a[ixj];
          const bool up = (i & k) == 0;
          if ((x > y) == up) {
            a[i] = y;
            a[ixj] = x;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Candidate mode (keys != NULL, row-sharded problems): instead of seeding, the
// min(n_empty, n) worst local points are written, worst first, as
// (key ^ 2^63, vector) with the point's global index (gofs[b] + i) in the key,
// for a cross-rank merge.
struct ReseedCand {
  const int64_t* gofs;
  int m_max;
  int64_t* keys;  // [nblk][m_max], pre-filled with INT64_MAX
  float* vecs;    // [nblk][m_max][bs]
};

__global__ void __launch_bounds__(RS_THREADS)
reseed_kernel(int metric, const float* __restrict__ X, const float* __restrict__ C,
              const int32_t* __restrict__ labels, int nblk, int n_pad, int k_pad, int bs,
              const int32_t* __restrict__ n, const int32_t* __restrict__ kvec, const int32_t* __restrict__ active,
              float* __restrict__ sums, const int32_t* __restrict__ counts, int32_t* __restrict__ n_empty_out,
              uint8_t* scratch, int k_pow2, int* err, ReseedCand cand) {
  __shared__ uint64_t s_sort[RS_SMEM_SORT];
  __shared__ int s_hist[256];
  __shared__ uint64_t s_prefix;
  __shared__ int s_need, s_done, s_count;
  int32_t* empty_ids = reinterpret_cast<int32_t*>(scratch + (size_t)blockIdx.x * ((size_t)k_pad * 4 + (size_t)k_pow2 * 8));
  uint64_t* g_list = reinterpret_cast<uint64_t*>(empty_ids + k_pad);
  for (int b = blockIdx.x; b < nblk; b += gridDim.x) {
    if (active && !active[b]) continue;
    const int nb = n[b], kb = kvec[b];
    const int32_t* cnt = counts + (int64_t)b * k_pad;
    // 1. empty clusters, ascending
    int n_empty = 0;
    for (int c0 = 0; c0 < kb; c0 += blockDim.x) {
      const int c = c0 + threadIdx.x;
      const int e = (c < kb && cnt[c] == 0) ? 1 : 0;
      int tot;
      const int pos = block_exclusive_scan(e, &tot);
      if (e) empty_ids[n_empty + pos] = c;
      n_empty += tot;
    }
    if (threadIdx.x == 0) n_empty_out[b] = n_empty;
    const int n_sel = cand.keys ? min(n_empty, nb) : n_empty;
    if (n_sel == 0) continue;
    const uint32_t gofs = cand.keys ? (uint32_t)cand.gofs[b] : 0u;
    const float* Xb = X + (int64_t)b * n_pad * bs;
    const float* Cb = C + (int64_t)b * k_pad * bs;
    const int32_t* Lb = labels + (int64_t)b * n_pad;
    // 2. radix select of the n_empty smallest (score-key, point) composites
    if (threadIdx.x == 0) {
      s_prefix = 0;
      s_need = n_sel;
      s_done = 0;
    }
    __syncthreads();
    uint64_t thresh = ~0ull;
    for (int shift = 56; shift >= 0; shift -= 8) {
      for (int t = threadIdx.x; t < 256; t += blockDim.x) s_hist[t] = 0;
      __syncthreads();
      const uint64_t hmask = shift == 56 ? 0ull : (~0ull << (shift + 8));
      const uint64_t pref = s_prefix;
      for (int i = threadIdx.x; i < nb; i += blockDim.x) {
        const uint64_t key = reseed_key(metric, Xb + (int64_t)i * bs, Cb + (int64_t)Lb[i] * bs, bs, gofs + i);
        if ((key & hmask) == (pref & hmask)) atomicAdd(&s_hist[(key >> shift) & 255], 1);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        int need = s_need, cum = 0, d = 0;
        for (; d < 255; ++d) {
          if (cum + s_hist[d] >= need) break;
          cum += s_hist[d];
        }
        need -= cum;
        s_prefix = pref | ((uint64_t)d << shift);
        s_need = need;
        if (s_hist[d] == need) s_done = 1;  // every key under this prefix is selected
      }
      __syncthreads();
      if (s_done) {
        thresh = s_prefix | (shift == 0 ? 0ull : ((1ull << shift) - 1));
        break;
      }
      if (shift == 0) thresh = s_prefix;
    }
    // 3. collect the selected composites
    int m_pow2 = 1;
    while (m_pow2 < n_sel) m_pow2 <<= 1;
    uint64_t* list = m_pow2 <= RS_SMEM_SORT ? s_sort : g_list;
    if (threadIdx.x == 0) s_count = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < m_pow2; i += blockDim.x) list[i] = ~0ull;
    __syncthreads();
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
      const uint64_t key = reseed_key(metric, Xb + (int64_t)i * bs, Cb + (int64_t)Lb[i] * bs, bs, gofs + i);
      if (key <= thresh) {
        const int pos = atomicAdd(&s_count, 1);
        if (pos < m_pow2) list[pos] = key;
      }
    }
    __syncthreads();
    if (s_count != n_sel) {
      if (threadIdx.x == 0) atomicCAS(err, 0, 21);
      __syncthreads();
      continue;
    }
    // 4. order them (ascending key = worst first)
    bitonic_sort(list, m_pow2);
    if (cand.keys) {
      for (int t = threadIdx.x; t < n_sel * bs; t += blockDim.x) {
        const int e = t / bs, j = t - e * bs;
        const uint32_t row = (uint32_t)(list[e] & 0xffffffffu) - gofs;
        cand.vecs[((int64_t)b * cand.m_max + e) * bs + j] = Xb[(int64_t)row * bs + j];
        if (j == 0) cand.keys[(int64_t)b * cand.m_max + e] = (int64_t)(list[e] ^ (1ull << 63));
      }
      __syncthreads();
      continue;
    }
    // 5. the i-th worst point seeds the i-th empty cluster
    float* Sb = sums + (int64_t)b * k_pad * bs;
    for (int t = threadIdx.x; t < n_empty * bs; t += blockDim.x) {
      const int e = t / bs, j = t - e * bs;
      const uint32_t row = (uint32_t)(list[e] & 0xffffffffu);
      Sb[(int64_t)empty_ids[e] * bs + j] = Xb[(int64_t)row * bs + j];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Finalize
// ---------------------------------------------------------------------------

__global__ void finalize_kernel(int metric, float* __restrict__ sums, int32_t* __restrict__ counts,
                                const int32_t* __restrict__ n_empty, int nblk, int k_pad, int bs,
                                const int32_t* __restrict__ kvec, int32_t* __restrict__ active,
                                int32_t* __restrict__ converged, int32_t* __restrict__ iters_run,
                                float* __restrict__ moved_hist, int32_t* __restrict__ nempty_hist, int iter,
                                float* __restrict__ C, uint8_t* __restrict__ changed) {
  for (int b = blockIdx.x; b < nblk; b += gridDim.x) {
    if (!active[b]) continue;
    const int kb = kvec[b];
    float* Sb = sums + (int64_t)b * k_pad * bs;
    int32_t* Nb = counts + (int64_t)b * k_pad;
    float* Cb = C + (int64_t)b * k_pad * bs;
    float part = 0.f;
    for (int c = threadIdx.x; c < kb; c += blockDim.x) {
      float* s = Sb + (int64_t)c * bs;
      float* cc = Cb + (int64_t)c * bs;
      const int cnt = Nb[c];
      if (changed) {
        uint8_t& ch = changed[(int64_t)b * k_pad + c];
        if (cnt > 0 && !ch) {
          // same members as at the previous update: the same centroid, kept bit for bit
          for (int j = 0; j < bs; ++j) s[j] = 0.f;
          Nb[c] = 0;
          continue;
        }
      }
      float den;
      if (metric == SKCQ_METRIC_COSINE) {
        float q = 0.f;
        for (int j = 0; j < bs; ++j) q = __fmaf_rn(s[j], s[j], q);
        den = fmaxf(sqrtf(q), 1e-12f);  // F.normalize
      } else {
        den = cnt > 0 ? (float)cnt : 1.f;  // reseeded clusters keep the point
      }
      bool differs = false;
      for (int j = 0; j < bs; ++j) {
        const float nv = (metric == SKCQ_METRIC_COSINE || cnt > 0) ? __fdiv_rn(s[j], den) : s[j];
        const float d = __fsub_rn(nv, cc[j]);
        part = __fmaf_rn(d, d, part);
        differs |= __float_as_uint(nv) != __float_as_uint(cc[j]);
        cc[j] = nv;
        s[j] = 0.f;
      }
      Nb[c] = 0;
      // recomputed (or reseeded): moved for the next assignment unless the
      // value came out bit for bit the same (e.g. a Forgy seed alone in its cluster)
      if (changed) changed[(int64_t)b * k_pad + c] = differs ? 1 : 0;
    }
    const float tot = block_sum(part);
    if (threadIdx.x == 0) {
      const float moved = sqrtf(tot);
      moved_hist[(int64_t)iter * nblk + b] = moved;
      nempty_hist[(int64_t)iter * nblk + b] = n_empty[b];
      iters_run[b] = iter + 1;
      if (moved < 1e-6f) {
        active[b] = 0;
        converged[b] = 1;
      }
    }
    __syncthreads();
  }
}

// Rows of BS floats (16-, 8- or 4-byte vectors; a row starts at a multiple of
// BS * 4 bytes of a 16-byte aligned problem slice).
template <int BS>
__device__ __forceinline__ void fin_load(const float* p, float (&v)[BS]) {
  if constexpr (BS % 4 == 0) {
#pragma unroll
    for (int i = 0; i < BS / 4; ++i) {
      const float4 t = reinterpret_cast<const float4*>(p)[i];
      v[4 * i] = t.x, v[4 * i + 1] = t.y, v[4 * i + 2] = t.z, v[4 * i + 3] = t.w;
    }
  } else if constexpr (BS % 2 == 0) {
#pragma unroll
    for (int i = 0; i < BS / 2; ++i) {
      const float2 t = reinterpret_cast<const float2*>(p)[i];
      v[2 * i] = t.x, v[2 * i + 1] = t.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < BS; ++i) v[i] = p[i];
  }
}

template <int BS>
__device__ __forceinline__ void fin_store(float* p, const float (&v)[BS]) {
  if constexpr (BS % 4 == 0) {
#pragma unroll
    for (int i = 0; i < BS / 4; ++i)
      reinterpret_cast<float4*>(p)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  } else if constexpr (BS % 2 == 0) {
#pragma unroll
    for (int i = 0; i < BS / 2; ++i) reinterpret_cast<float2*>(p)[i] = make_float2(v[2 * i], v[2 * i + 1]);
  } else {
#pragma unroll
    for (int i = 0; i < BS; ++i) p[i] = v[i];
  }
}

// finalize_kernel for a compile-time block size: the same arithmetic, and the
// same centroids per thread in the same order (so `moved` has the same bits),
// with each row moved as vectors and fin_unroll<BS>() centroids in flight per
// thread. A cluster that kept its members (cnt > 0, not changed) has its sum
// row zeroed without being read, and its centroid row is not touched.
constexpr int FIN_THREADS = 256;
template <int BS>
__host__ __device__ constexpr int fin_unroll() {
  return BS >= 12 ? 2 : 4;
}

template <int BS>
__global__ void __launch_bounds__(FIN_THREADS) finalize_vec_kernel(
    int metric, float* __restrict__ sums, int32_t* __restrict__ counts, const int32_t* __restrict__ n_empty, int nblk,
    int k_pad, const int32_t* __restrict__ kvec, int32_t* __restrict__ active, int32_t* __restrict__ converged,
    int32_t* __restrict__ iters_run, float* __restrict__ moved_hist, int32_t* __restrict__ nempty_hist, int iter,
    float* __restrict__ C, uint8_t* __restrict__ changed) {
  for (int b = blockIdx.x; b < nblk; b += gridDim.x) {
    if (!active[b]) continue;
    const int kb = kvec[b];
    float* Sb = sums + (int64_t)b * k_pad * BS;
    int32_t* Nb = counts + (int64_t)b * k_pad;
    float* Cb = C + (int64_t)b * k_pad * BS;
    uint8_t* chb = changed ? changed + (int64_t)b * k_pad : nullptr;
    float part = 0.f;
    constexpr int FIN_UNROLL = fin_unroll<BS>();
    for (int c0 = threadIdx.x; c0 < kb; c0 += FIN_UNROLL * FIN_THREADS) {
      int cnt[FIN_UNROLL];
      bool redo[FIN_UNROLL];
#pragma unroll
      for (int u = 0; u < FIN_UNROLL; ++u) {
        const int c = c0 + u * FIN_THREADS;
        cnt[u] = c < kb ? Nb[c] : 0;
        redo[u] = c < kb && !(chb && cnt[u] > 0 && !chb[c]);
      }
      float s[FIN_UNROLL][BS], cv[FIN_UNROLL][BS];
#pragma unroll
      for (int u = 0; u < FIN_UNROLL; ++u) {
        const int c = c0 + u * FIN_THREADS;
        if (redo[u]) {
          fin_load<BS>(Sb + (int64_t)c * BS, s[u]);
          fin_load<BS>(Cb + (int64_t)c * BS, cv[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < FIN_UNROLL; ++u) {
        const int c = c0 + u * FIN_THREADS;
        if (c >= kb) continue;
        float z[BS];
#pragma unroll
        for (int j = 0; j < BS; ++j) z[j] = 0.f;
        fin_store<BS>(Sb + (int64_t)c * BS, z);
        Nb[c] = 0;
        // same members as at the previous update: the same centroid, kept bit for bit
        if (!redo[u]) continue;
        float den;
        if (metric == SKCQ_METRIC_COSINE) {
          float q = 0.f;
#pragma unroll
          for (int j = 0; j < BS; ++j) q = __fmaf_rn(s[u][j], s[u][j], q);
          den = fmaxf(sqrtf(q), 1e-12f);  // F.normalize
        } else {
          den = cnt[u] > 0 ? (float)cnt[u] : 1.f;  // reseeded clusters keep the point
        }
        bool differs = false;
#pragma unroll
        for (int j = 0; j < BS; ++j) {
          const float nv = (metric == SKCQ_METRIC_COSINE || cnt[u] > 0) ? __fdiv_rn(s[u][j], den) : s[u][j];
          const float d = __fsub_rn(nv, cv[u][j]);
          part = __fmaf_rn(d, d, part);
          differs |= __float_as_uint(nv) != __float_as_uint(cv[u][j]);
          cv[u][j] = nv;
        }
        fin_store<BS>(Cb + (int64_t)c * BS, cv[u]);
        // recomputed (or reseeded): moved for the next assignment unless the
        // value came out bit for bit the same (e.g. a Forgy seed alone in its cluster)
        if (chb) chb[c] = differs ? 1 : 0;
      }
    }
    const float tot = block_sum(part);
    if (threadIdx.x == 0) {
      const float moved = sqrtf(tot);
      moved_hist[(int64_t)iter * nblk + b] = moved;
      nempty_hist[(int64_t)iter * nblk + b] = n_empty[b];
      iters_run[b] = iter + 1;
      if (moved < 1e-6f) {
        active[b] = 0;
        converged[b] = 1;
      }
    }
    __syncthreads();
  }
}

}  // namespace skcq

using namespace skcq;

extern "C" int skcq_update(const float* R, const int32_t* labels, int nblk, int n_pad, int k_pad, int bs,
                             const int32_t* n, const int32_t* k, const int32_t* active, float* sums,
                             int32_t* counts, const uint8_t* changed, void* stream) {
  SKCQ_REQUIRE(R && labels && n && k && sums && counts, SKCQ_ERR_INVALID, "update: null pointer");
  SKCQ_REQUIRE(bs > 0 && bs <= 64, SKCQ_ERR_INVALID, "update: bad block size %d", bs);
  cudaStream_t s = (cudaStream_t)stream;
  // columns per pass: all bs if a cluster row fits, else the widest split that does
  int cpp = bs;
  while (cpp > 1 && (size_t)k_pad * update_row_stride(cpp) * sizeof(float) > (size_t)UPDATE_SMEM) cpp = (cpp + 1) / 2;
  const size_t smem = (size_t)k_pad * update_row_stride(cpp) * sizeof(float);
  const int passes = (bs + cpp - 1) / cpp;
  if (smem <= (size_t)UPDATE_SMEM && nblk <= 65535 && passes <= 8) {
    static thread_local int configured_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_dev != dev) {
      cudaError_t e = cudaFuncSetAttribute(update_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, UPDATE_SMEM);
      if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "update: %s", cudaGetErrorString(e));
      configured_dev = dev;
    }
    // enough CTAs to fill the machine, each with at least 4 rows per accumulator entry
    int64_t rows = (int64_t)nblk * n_pad;
    int64_t target = 148 * 2;
    int64_t rpc = (rows + target - 1) / target;
    int64_t min_rpc = (int64_t)k_pad * 4;
    if (rpc < min_rpc) rpc = min_rpc;
    if (rpc > n_pad) rpc = n_pad;
    dim3 grid((unsigned)((n_pad + rpc - 1) / rpc), nblk, passes);
    update_smem_kernel<<<grid, 512, smem, s>>>(R, labels, n_pad, k_pad, bs, cpp, n, active, k, (int)rpc, sums,
                                               counts, changed);
    return check_launch("update (shared)");
  }
  int64_t work = (int64_t)nblk * n_pad;
  int grid = (int)((work + 255) / 256);
  if (grid > 148 * 32) grid = 148 * 32;
  update_global_kernel<<<grid, 256, 0, s>>>(R, labels, nblk, n_pad, k_pad, bs, n, active, sums, counts, changed);
  return check_launch("update (global)");
}

// Largest centroid count a reseed accepts (the reseed's per-problem scratch
// holds k_pad ids and a pow2(k_pad) sort list; beyond this the int arithmetic
// below would overflow).
constexpr int RESEED_MAX_KPAD = 1 << 20;

static int pow2_at_least(int v) {
  int p = 1;
  while (p < v && p < RESEED_MAX_KPAD) p <<= 1;
  return p;
}

static int reseed_grid(int nblk) { return nblk < 296 ? nblk : 296; }

extern "C" size_t skcq_reseed_scratch_bytes(int nblk, int k_pad) {
  if (nblk <= 0 || k_pad <= 0 || k_pad > RESEED_MAX_KPAD) return 0;
  return (size_t)reseed_grid(nblk) * ((size_t)k_pad * 4 + (size_t)pow2_at_least(k_pad) * 8);
}

extern "C" int skcq_reseed(int metric, const float* X, const float* C, const int32_t* labels, int nblk, int n_pad,
                           int k_pad, int bs, const int32_t* n, const int32_t* k, const int32_t* active, float* sums,
                           const int32_t* counts, int32_t* n_empty, void* scratch, void* stream) {
  SKCQ_REQUIRE(X && C && labels && n && k && sums && counts && n_empty && scratch, SKCQ_ERR_INVALID,
               "reseed: null pointer");
  SKCQ_REQUIRE(bs > 0 && bs <= 64, SKCQ_ERR_INVALID, "reseed: bad block size %d", bs);
  SKCQ_REQUIRE(k_pad > 0 && k_pad <= RESEED_MAX_KPAD && k_pad % SKCQ_CENT_TILE == 0, SKCQ_ERR_INVALID,
               "reseed: k_pad %d must be a positive multiple of %d, at most %d", k_pad, SKCQ_CENT_TILE,
               RESEED_MAX_KPAD);
  SKCQ_REQUIRE(((uintptr_t)scratch & 7) == 0, SKCQ_ERR_INVALID, "reseed: scratch must be 8-byte aligned");
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "reseed: no device error word");
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(n_empty, 0, sizeof(int32_t) * nblk, s);
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "reseed: %s", cudaGetErrorString(e));
  reseed_kernel<<<reseed_grid(nblk), RS_THREADS, 0, s>>>(metric, X, C, labels, nblk, n_pad, k_pad, bs, n, k, active,
                                                         sums, counts, n_empty, (uint8_t*)scratch,
                                                         pow2_at_least(k_pad), err, ReseedCand{});
  return check_launch("reseed");
}

extern "C" int skcq_reseed_candidates(int metric, const float* X, const float* C, const int32_t* labels, int nblk,
                                      int n_pad, int k_pad, int bs, const int32_t* n, const int32_t* k,
                                      const int32_t* active, const int32_t* counts, const int64_t* gofs, int m_max,
                                      int64_t* keys, float* vecs, int32_t* n_empty, void* scratch, void* stream) {
  SKCQ_REQUIRE(X && C && labels && n && k && counts && gofs && keys && vecs && n_empty && scratch, SKCQ_ERR_INVALID,
               "reseed_candidates: null pointer");
  SKCQ_REQUIRE(bs > 0 && bs <= 64 && m_max > 0, SKCQ_ERR_INVALID, "reseed_candidates: bs %d, m_max %d", bs, m_max);
  SKCQ_REQUIRE(k_pad > 0 && k_pad <= RESEED_MAX_KPAD && k_pad % SKCQ_CENT_TILE == 0, SKCQ_ERR_INVALID,
               "reseed_candidates: k_pad %d must be a positive multiple of %d, at most %d", k_pad, SKCQ_CENT_TILE,
               RESEED_MAX_KPAD);
  SKCQ_REQUIRE(((uintptr_t)scratch & 7) == 0, SKCQ_ERR_INVALID, "reseed_candidates: scratch must be 8-byte aligned");
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "reseed_candidates: no device error word");
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(n_empty, 0, sizeof(int32_t) * nblk, s);
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "reseed_candidates: %s", cudaGetErrorString(e));
  reseed_kernel<<<reseed_grid(nblk), RS_THREADS, 0, s>>>(metric, X, C, labels, nblk, n_pad, k_pad, bs, n, k, active,
                                                         nullptr, counts, n_empty, (uint8_t*)scratch,
                                                         pow2_at_least(k_pad), err,
                                                         ReseedCand{gofs, m_max, keys, vecs});
  return check_launch("reseed_candidates");
}

extern "C" int skcq_finalize(int metric, float* sums, int32_t* counts, const int32_t* n_empty, int nblk, int k_pad,
                             int bs, const int32_t* k, int32_t* active, int32_t* converged, int32_t* iters_run,
                             float* moved_hist, int32_t* nempty_hist, int iter, float* C, uint8_t* changed,
                             void* stream) {
  SKCQ_REQUIRE(sums && counts && n_empty && k && active && converged && iters_run && moved_hist && nempty_hist && C,
               SKCQ_ERR_INVALID, "finalize: null pointer");
  int grid = nblk < 1024 ? nblk : 1024;
  if (grid == 0) return SKCQ_OK;
  using VecFn = void (*)(int, float*, int32_t*, const int32_t*, int, int, const int32_t*, int32_t*, int32_t*,
                         int32_t*, float*, int32_t*, int, float*, uint8_t*);
  VecFn vec = nullptr;
  switch (bs) {
    case 4: vec = finalize_vec_kernel<4>; break;
    case 6: vec = finalize_vec_kernel<6>; break;
    case 8: vec = finalize_vec_kernel<8>; break;
    case 12: vec = finalize_vec_kernel<12>; break;
    case 16: vec = finalize_vec_kernel<16>; break;
    default: break;
  }
  const bool aligned = (((uintptr_t)sums | (uintptr_t)C) & 15) == 0 && k_pad % 4 == 0;
  if (vec && aligned) {
    vec<<<grid, FIN_THREADS, 0, (cudaStream_t)stream>>>(metric, sums, counts, n_empty, nblk, k_pad, k, active,
                                                        converged, iters_run, moved_hist, nempty_hist, iter, C,
                                                        changed);
    return check_launch("finalize");
  }
  finalize_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(metric, sums, counts, n_empty, nblk, k_pad, bs, k, active,
                                                          converged, iters_run, moved_hist, nempty_hist, iter, C,
                                                          changed);
  return check_launch("finalize");
}

// ---------------------------------------------------------------------------
// Allocation-free reseed
//
// skcq_reseed needs a caller-provided scratch buffer. Some callers cannot
// obtain one: a host runtime that has already handed all device memory to its
// own allocator and forbids further cudaMalloc, or a plug-in whose host
// interface only passes it the input and output buffers of the step. For them
// skcq_reseed_noalloc keeps the scratch in a fixed device array compiled into
// this library (RESEED_STATIC_BYTES on every GPU that loads the library, held
// until the process exits) and allocates nothing.
// ---------------------------------------------------------------------------

constexpr size_t RESEED_STATIC_BYTES = (size_t)16 << 20;  // 16 MiB per device
static __device__ __align__(256) uint8_t g_reseed_scratch[RESEED_STATIC_BYTES];

// Device address of g_reseed_scratch on the current device. The host-side
// symbol is only a stand-in, so the address is looked up once per device (with
// that device current) and cached for the life of the process. The cache is
// not refreshed after cudaDeviceReset (or any re-creation of the device's
// primary context): the entry point must not be used across a device reset.
static int reseed_static_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "reseed_noalloc: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(SKCQ_ERR_INVALID, "reseed_noalloc: device ordinal %d >= 64", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_reseed_scratch);
    if (e != cudaSuccess || p == nullptr)
      return set_error(SKCQ_ERR_CUDA, "reseed_noalloc: cannot resolve the static scratch (%s)", cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return SKCQ_OK;
}

extern "C" int skcq_reseed_noalloc(int metric, const float* X, const float* C, const int32_t* labels, int nblk,
                                   int n_pad, int k_pad, int bs, const int32_t* n, const int32_t* k,
                                   const int32_t* active, float* sums, const int32_t* counts, int32_t* n_empty,
                                   void* stream) {
  SKCQ_REQUIRE(X && C && labels && n && k && sums && counts && n_empty, SKCQ_ERR_INVALID,
               "reseed_noalloc: null pointer");
  SKCQ_REQUIRE(bs > 0 && bs <= 64, SKCQ_ERR_INVALID, "reseed_noalloc: bad block size %d", bs);
  SKCQ_REQUIRE(nblk > 0 && k_pad > 0, SKCQ_ERR_INVALID, "reseed_noalloc: empty problem set");
  SKCQ_REQUIRE(k_pad % SKCQ_CENT_TILE == 0, SKCQ_ERR_INVALID, "reseed_noalloc: k_pad %d not a multiple of %d", k_pad,
               SKCQ_CENT_TILE);
  SKCQ_REQUIRE(k_pad <= RESEED_MAX_KPAD, SKCQ_ERR_INVALID,
               "reseed_noalloc: k_pad %d over the static buffer's limit of %d centroids per problem; use "
               "skcq_reseed with caller scratch",
               k_pad, RESEED_MAX_KPAD);
  const size_t per_slot = (size_t)k_pad * 4 + (size_t)pow2_at_least(k_pad) * 8;
  SKCQ_REQUIRE(per_slot <= RESEED_STATIC_BYTES, SKCQ_ERR_INVALID,
               "reseed_noalloc: k_pad %d needs %zu scratch bytes per problem, over the %zu-byte static buffer "
               "(at most 1048576 centroids per problem); use skcq_reseed with caller scratch",
               k_pad, per_slot, RESEED_STATIC_BYTES);
  void* scratch = nullptr;
  int rc = reseed_static_scratch(&scratch);
  if (rc != SKCQ_OK) return rc;
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "reseed_noalloc: no device error word");
  // Fewer concurrent problems when they do not all fit: CTAs stride over the set.
  int grid = reseed_grid(nblk);
  const int fit = (int)(RESEED_STATIC_BYTES / per_slot);
  if (grid > fit) grid = fit;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(n_empty, 0, sizeof(int32_t) * nblk, s);
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "reseed_noalloc: %s", cudaGetErrorString(e));
  reseed_kernel<<<grid, RS_THREADS, 0, s>>>(metric, X, C, labels, nblk, n_pad, k_pad, bs, n, k, active, sums, counts,
                                           n_empty, (uint8_t*)scratch, pow2_at_least(k_pad), err, ReseedCand{});
  return check_launch("reseed_noalloc");
}
