// Incremental Lloyd assignment: after the first iterations most clusters keep
// their members, so most centroids keep their exact value, and a point's
// nearest centroid can only change if its own centroid moved or a moved
// centroid now beats it.
//
// Exactness. The Lloyd update (kmeans.py:152-188, 210-244) computes each
// centroid from its members only, so a cluster whose member set did not change
// since the previous update gets the same value again; skcq_finalize with a
// `changed` mask keeps such centroids bit for bit. With X and those centroids
// unchanged, every score of an unmoved centroid is bit-identical to the
// previous assignment's, so for a point whose assigned centroid a did not
// move, the new arg-max over all K centroids (first maximum wins) is a, or the
// best moved centroid if that one scores higher, or scores the same with a
// lower index. Points whose own centroid moved are re-assigned over all K.
//
// Kernels here:
//   mark_changed   changed[b][c] = 1 for every cluster that gained or lost a
//                  point between two assignments (or all, on the first)
//   moved_lists    ascending lists of the moved centroids and of the points
//                  assigned to one, per problem
//   gather_rows    dst[b][j] = src[b][idx[b][j]] (moved centroids, flagged points)
//   assign_merge   per point: keep a, or take the best moved centroid, or the
//                  full re-assignment of a flagged point
// The two tensor-core passes in between (moved centroids for all points; all
// centroids for the flagged points) are skcq_assign calls by the host.
#include "common.cuh"

namespace skcq {

constexpr int MC_THREADS = 256;
constexpr int CP_THREADS = 1024;
constexpr int CP_ITEMS = 4;  // consecutive items per thread
constexpr int CP_CHUNK = CP_THREADS * CP_ITEMS;

__global__ void mark_reset_kernel(int nblk, int k_pad, const int32_t* __restrict__ mask, int all,
                                  uint8_t* __restrict__ changed) {
  const int b = blockIdx.y;
  if (mask && !mask[b]) return;
  uint8_t* row = changed + (int64_t)b * k_pad;
  for (int c = blockIdx.x * MC_THREADS + threadIdx.x; c < k_pad; c += gridDim.x * MC_THREADS) row[c] = all ? 1 : 0;
}

__global__ void mark_diff_kernel(const int32_t* __restrict__ prev, const int32_t* __restrict__ labels, int n_pad,
                                 int k_pad, const int32_t* __restrict__ n, const int32_t* __restrict__ mask,
                                 uint8_t* __restrict__ changed, int* err) {
  const int b = blockIdx.y;
  if (mask && !mask[b]) return;
  const int nb = n[b];
  uint8_t* row = changed + (int64_t)b * k_pad;
  const int32_t* P = prev + (int64_t)b * n_pad;
  const int32_t* L = labels + (int64_t)b * n_pad;
  for (int i = blockIdx.x * MC_THREADS + threadIdx.x; i < nb; i += gridDim.x * MC_THREADS) {
    const int p = P[i], l = L[i];
    if (p == l) continue;
    if (p < 0 || p >= k_pad || l < 0 || l >= k_pad) {
      atomicCAS(err, 0, 71);
      continue;
    }
    row[p] = 1;  // plain stores of the same value: no ordering needed
    row[l] = 1;
  }
}

// flag of item i of problem b: centroid lists (which == 0), points whose
// centroid moved (1), or points marked in a per-point array (2, `changed` then
// being [nblk][n_pad])
__device__ __forceinline__ bool cp_flag(int which, int b, int i, int n_pad, int k_pad, const int32_t* n,
                                        const int32_t* k, const uint8_t* changed, const int32_t* labels) {
  if (which == 2) return i < n[b] && changed[(int64_t)b * n_pad + i];
  const uint8_t* row = changed + (int64_t)b * k_pad;
  if (which == 0) return i < k[b] && row[i];
  if (i >= n[b]) return false;
  const int l = labels[(int64_t)b * n_pad + i];
  return l >= 0 && l < k_pad && row[l];
}

// cnt[b][chunk] = flagged items of the chunk
__global__ void __launch_bounds__(CP_THREADS) cp_count_kernel(int which, int items, int n_pad, int k_pad,
                                                              const int32_t* __restrict__ n,
                                                              const int32_t* __restrict__ k,
                                                              const int32_t* __restrict__ mask,
                                                              const uint8_t* __restrict__ changed,
                                                              const int32_t* __restrict__ labels, int n_chunks,
                                                              int32_t* __restrict__ cnt) {
  const int b = blockIdx.y;
  if (mask && !mask[b]) return;
  const int i0 = blockIdx.x * CP_CHUNK + threadIdx.x * CP_ITEMS;
  int c = 0;
#pragma unroll
  for (int j = 0; j < CP_ITEMS; ++j)
    if (i0 + j < items && cp_flag(which, b, i0 + j, n_pad, k_pad, n, k, changed, labels)) ++c;
  int tot;
  block_exclusive_scan(c, &tot);
  if (threadIdx.x == 0) cnt[(int64_t)b * n_chunks + blockIdx.x] = tot;
}

// list[b][pos] = i for the flagged items in ascending order; count[b] = total
__global__ void __launch_bounds__(CP_THREADS) cp_place_kernel(int which, int items, int n_pad, int k_pad,
                                                              const int32_t* __restrict__ n,
                                                              const int32_t* __restrict__ k,
                                                              const int32_t* __restrict__ mask,
                                                              const uint8_t* __restrict__ changed,
                                                              const int32_t* __restrict__ labels, int n_chunks,
                                                              const int32_t* __restrict__ cnt, int list_ld,
                                                              int32_t* __restrict__ list, int32_t* __restrict__ count) {
  __shared__ int s_base;
  const int b = blockIdx.y;
  if (mask && !mask[b]) return;
  if (threadIdx.x == 0) {
    int s = 0;
    for (int c = 0; c < (int)blockIdx.x; ++c) s += cnt[(int64_t)b * n_chunks + c];
    s_base = s;
  }
  const int i0 = blockIdx.x * CP_CHUNK + threadIdx.x * CP_ITEMS;
  bool f[CP_ITEMS];
  int c = 0;
#pragma unroll
  for (int j = 0; j < CP_ITEMS; ++j) {
    f[j] = i0 + j < items && cp_flag(which, b, i0 + j, n_pad, k_pad, n, k, changed, labels);
    c += f[j] ? 1 : 0;
  }
  int tot;
  const int off = block_exclusive_scan(c, &tot);  // synchronises, so s_base is visible
  int pos = s_base + off;
  int32_t* out = list + (int64_t)b * list_ld;
#pragma unroll
  for (int j = 0; j < CP_ITEMS; ++j)
    if (f[j]) out[pos++] = i0 + j;
  if (blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) count[b] = s_base + tot;
}

__global__ void gather_rows_kernel(const float* __restrict__ src, int src_rows, const int32_t* __restrict__ idx,
                                   int idx_ld, const int32_t* __restrict__ count, int out_rows, int bs,
                                   float* __restrict__ dst, int* err) {
  const int b = blockIdx.y;
  const int cb = count[b];
  const float* S = src + (int64_t)b * src_rows * bs;
  float* D = dst + (int64_t)b * out_rows * bs;
  const int64_t total = (int64_t)out_rows * bs;
  for (int64_t e = blockIdx.x * (int64_t)MC_THREADS + threadIdx.x; e < total; e += (int64_t)gridDim.x * MC_THREADS) {
    const int j = (int)(e / bs), d = (int)(e - (int64_t)j * bs);
    float v = 0.f;
    if (j < cb) {
      const int r = idx[(int64_t)b * idx_ld + j];
      if (r >= 0 && r < src_rows)
        v = S[(int64_t)r * bs + d];
      else
        atomicCAS(err, 0, 72);
    }
    D[e] = v;
  }
}

// The reference score of point x against centroid c, computed exactly as the
// assignment's re-score does (sequential FMAs; euclidean -(||c||^2 - 2 x.c)),
// NaN as -inf and -0 as +0.
__device__ __forceinline__ uint32_t exact_key(int metric, const float* x, const float* c, float cn, int bs) {
  float dot = 0.f;
  for (int j = 0; j < bs; ++j) dot = __fmaf_rn(x[j], c[j], dot);
  float sc = metric == SKCQ_METRIC_COSINE ? dot : -__fadd_rn(__fmul_rn(dot, -2.0f), cn);
  if (sc != sc) sc = -INFINITY;
  return float_key(sc + 0.0f);
}

__global__ void assign_merge_kernel(int metric, const float* __restrict__ X, const float* __restrict__ C,
                                    const float* __restrict__ cnorm, int n_pad, int k_pad, int bs,
                                    const int32_t* __restrict__ n, const int32_t* __restrict__ active,
                                    const uint8_t* __restrict__ changed, const int32_t* __restrict__ mlist,
                                    const int32_t* __restrict__ mcount, const int32_t* __restrict__ labels_m,
                                    const int32_t* __restrict__ plist, const int32_t* __restrict__ pcount, int p_pad,
                                    const int32_t* __restrict__ labels_f, int32_t* __restrict__ labels,
                                    const float* __restrict__ C_old, const float* __restrict__ cnorm_old,
                                    uint8_t* __restrict__ unres, int phase, int* err) {
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int nb = n[b], mb = mcount[b], pb = pcount[b];
  const uint8_t* row = changed + (int64_t)b * k_pad;
  const float* Xb = X + (int64_t)b * n_pad * bs;
  const float* Cb = C + (int64_t)b * k_pad * bs;
  const float* Nb = cnorm + (int64_t)b * k_pad;
  int32_t* Lb = labels + (int64_t)b * n_pad;
  uint8_t* Ub = unres ? unres + (int64_t)b * n_pad : nullptr;
  if ((phase == 0 && mb <= 0) || (phase == 1 && pb <= 0)) {  // nothing to merge in this phase
    if (phase == 0 && Ub)
      for (int i = blockIdx.x * MC_THREADS + threadIdx.x; i < nb; i += gridDim.x * MC_THREADS) Ub[i] = 0;
    return;
  }
  const int lim = nb > pb ? nb : pb;
  for (int i = blockIdx.x * MC_THREADS + threadIdx.x; i < lim; i += gridDim.x * MC_THREADS) {
    if (phase == 0 && i < nb) {
      const int a = Lb[i];
      if (Ub) Ub[i] = 0;
      if (a < 0 || a >= k_pad) {
        atomicCAS(err, 0, 73);
      } else if (row[a] && Ub) {
        // its centroid moved: the best moved centroid wins outright when it
        // scores above a's previous score (which bounds every unmoved
        // centroid's unchanged score); otherwise a full search
        const int w = labels_m[(int64_t)b * n_pad + i];
        const int cand = (w >= 0 && w < mb) ? mlist[(int64_t)b * k_pad + w] : -1;
        bool done = false;
        if (cand >= 0 && cand < k_pad) {
          const float* x = Xb + (int64_t)i * bs;
          const uint32_t ko = exact_key(metric, x, C_old + ((int64_t)b * k_pad + a) * bs,
                                        cnorm_old[(int64_t)b * k_pad + a], bs);
          const uint32_t kc = exact_key(metric, x, Cb + (int64_t)cand * bs, Nb[cand], bs);
          if (kc > ko) {
            Lb[i] = cand;
            done = true;
          }
        }
        if (!done) Ub[i] = 1;
      } else if (!row[a] && mb > 0) {
        const int w = labels_m[(int64_t)b * n_pad + i];
        if (w < 0) {
          // not scored against the moved centroids (exactly on its centroid): keeps a
        } else if (w >= mb) {
          atomicCAS(err, 0, 74);
        } else {
          const int cand = mlist[(int64_t)b * k_pad + w];
          if (cand < 0 || cand >= k_pad) {
            atomicCAS(err, 0, 74);
          } else {
            const float* x = Xb + (int64_t)i * bs;
            const uint32_t ka = exact_key(metric, x, Cb + (int64_t)a * bs, Nb[a], bs);
            const uint32_t kc = exact_key(metric, x, Cb + (int64_t)cand * bs, Nb[cand], bs);
            if (kc > ka || (kc == ka && cand < a)) Lb[i] = cand;
          }
        }
      }
    }
    if (phase == 1 && i < pb) {  // a point whose centroid moved: its full re-assignment
      const int r = plist[(int64_t)b * n_pad + i];
      if (r < 0 || r >= nb)
        atomicCAS(err, 0, 75);
      else
        Lb[r] = labels_f[(int64_t)b * p_pad + i];
    }
  }
}

// Every unflagged point (its centroid a did not move) against the moved
// centroids of its problem, with the exact reference formula on CUDA cores:
// the list is staged in shared memory in slices of MX_SLICE centroids, each
// thread keeps the best (first maximum in list order, i.e. lowest index) and
// then compares it with a. For short moved lists this replaces the
// tensor-core pass over the gathered moved centroids and phase 0 of the merge.
constexpr int MX_SLICE = 256;
constexpr int MX_THREADS = 256;

template <int BS>
__global__ void __launch_bounds__(MX_THREADS) assign_moved_exact_kernel(
    int metric, const float* __restrict__ X, const float* __restrict__ C, const float* __restrict__ cnorm, int n_pad,
    int k_pad, int bs_rt, const int32_t* __restrict__ n, const int32_t* __restrict__ active,
    const uint8_t* __restrict__ changed, const int32_t* __restrict__ mlist, const int32_t* __restrict__ mcount,
    int32_t* __restrict__ labels, const float* __restrict__ C_old, const float* __restrict__ cnorm_old,
    uint8_t* __restrict__ unres, int* err) {
  constexpr int XN = BS > 0 ? BS : 32;
  const int bs = BS > 0 ? BS : bs_rt;
  extern __shared__ float sm[];
  float* tab = sm;                        // [MX_SLICE][bs]
  float* cn = sm + MX_SLICE * bs;         // [MX_SLICE]
  int* idx = reinterpret_cast<int*>(cn + MX_SLICE);  // [MX_SLICE]
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int nb = n[b], mb = mcount[b];
  uint8_t* Ub = unres ? unres + (int64_t)b * n_pad : nullptr;
  if (mb <= 0) {
    if (Ub)
      for (int i = blockIdx.x * MX_THREADS + threadIdx.x; i < nb; i += gridDim.x * MX_THREADS) Ub[i] = 0;
    return;
  }
  const uint8_t* row = changed + (int64_t)b * k_pad;
  const float* Cb = C + (int64_t)b * k_pad * bs;
  const float* Nb = cnorm + (int64_t)b * k_pad;
  const int32_t* Mb = mlist + (int64_t)b * k_pad;
  int32_t* Lb = labels + (int64_t)b * n_pad;
  for (int i0 = blockIdx.x * MX_THREADS; i0 < nb; i0 += gridDim.x * MX_THREADS) {
    const int i = i0 + threadIdx.x;
    int a = -1;
    bool moved_a = false;
    float x[XN];
    if (i < nb) {
      a = Lb[i];
      if (Ub) Ub[i] = 0;
      if (a < 0 || a >= k_pad) {
        atomicCAS(err, 0, 73);
        a = -1;
      } else if (row[a]) {
        moved_a = true;
        if (!Ub) a = -1;  // without the old scores: re-assigned over all centroids elsewhere
      }
    }
    if (a >= 0) {
#pragma unroll
      for (int j = 0; j < XN; ++j)
        if (BS > 0 || j < bs) x[j] = X[((int64_t)b * n_pad + i) * bs + j];
    }
    uint32_t best = 0;
    int best_c = -1;
    for (int s0 = 0; s0 < mb; s0 += MX_SLICE) {
      const int cnt = min(MX_SLICE, mb - s0);
      __syncthreads();
      for (int t = threadIdx.x; t < cnt; t += MX_THREADS) {
        int c = Mb[s0 + t];
        if (c < 0 || c >= k_pad) {
          atomicCAS(err, 0, 74);
          c = 0;
        }
        idx[t] = c;
        cn[t] = Nb[c];
      }
      __syncthreads();
      for (int e = threadIdx.x; e < cnt * bs; e += MX_THREADS) {
        const int t = e / bs, j = e - t * bs;
        tab[e] = Cb[(int64_t)idx[t] * bs + j];
      }
      __syncthreads();
      if (a >= 0) {
        for (int t = 0; t < cnt; ++t) {
          const float* c = tab + t * bs;
          float dot = 0.f;
#pragma unroll
          for (int j = 0; j < XN; ++j)
            if (BS > 0 || j < bs) dot = __fmaf_rn(x[j], c[j], dot);
          float sc = metric == SKCQ_METRIC_COSINE ? dot : -__fadd_rn(__fmul_rn(dot, -2.0f), cn[t]);
          if (sc != sc) sc = -INFINITY;
          const uint32_t key = float_key(sc + 0.0f);
          if (best_c < 0 || key > best) {
            best = key;
            best_c = idx[t];
          }
        }
      }
    }
    if (a >= 0 && best_c >= 0) {
      // unmoved a: its current score; moved a: its score before the update,
      // which bounds every unmoved centroid's (unchanged) score
      const float* ca = moved_a ? C_old + ((int64_t)b * k_pad + a) * bs : Cb + (int64_t)a * bs;
      const float na = moved_a ? cnorm_old[(int64_t)b * k_pad + a] : Nb[a];
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < XN; ++j)
        if (BS > 0 || j < bs) dot = __fmaf_rn(x[j], ca[j], dot);
      float sc = metric == SKCQ_METRIC_COSINE ? dot : -__fadd_rn(__fmul_rn(dot, -2.0f), na);
      if (sc != sc) sc = -INFINITY;
      const uint32_t ka = float_key(sc + 0.0f);
      if (moved_a) {
        if (best > ka)
          Lb[i] = best_c;
        else
          Ub[i] = 1;
      } else if (best > ka || (best == ka && best_c < a)) {
        Lb[i] = best_c;
      }
    } else if (moved_a && Ub) {
      Ub[i] = 1;
    }
  }
}

// Points the moved-centroid pass must score (euclidean): those whose centroid
// moved, and those not exactly on their centroid. A point equal to its
// unmoved centroid already has the largest score any centroid can reach
// (||c||^2 - 2 x.c = -||x||^2 + ||x - c||^2), so no moved centroid can beat it
// apart from one of identical value (an exact tie).
__global__ void mpass_points_kernel(const float* __restrict__ X, const float* __restrict__ C,
                                    const int32_t* __restrict__ labels, const uint8_t* __restrict__ changed,
                                    const int32_t* __restrict__ n, const int32_t* __restrict__ active, int n_pad,
                                    int k_pad, int bs, uint8_t* __restrict__ flags) {
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int nb = n[b];
  const float* Xb = X + (int64_t)b * n_pad * bs;
  const float* Cb = C + (int64_t)b * k_pad * bs;
  for (int i = blockIdx.x * MC_THREADS + threadIdx.x; i < nb; i += gridDim.x * MC_THREADS) {
    const int a = labels[(int64_t)b * n_pad + i];
    bool need = true;
    if (a >= 0 && a < k_pad && !changed[(int64_t)b * k_pad + a]) {
      need = false;
      for (int j = 0; j < bs; ++j)
        need |= __float_as_uint(Xb[(int64_t)i * bs + j]) != __float_as_uint(Cb[(int64_t)a * bs + j]);
    }
    flags[(int64_t)b * n_pad + i] = need ? 1 : 0;
  }
}

// labels_m[b][list[b][j]] = sub[b][j] for j < count[b]
__global__ void scatter_sub_kernel(const int32_t* __restrict__ list, const int32_t* __restrict__ count,
                                   const int32_t* __restrict__ sub, int s_pad, int n_pad,
                                   int32_t* __restrict__ labels_m, int* err) {
  const int b = blockIdx.y;
  const int cb = count[b];
  for (int j = blockIdx.x * MC_THREADS + threadIdx.x; j < cb && j < s_pad; j += gridDim.x * MC_THREADS) {
    const int i = list[(int64_t)b * n_pad + j];
    if (i < 0 || i >= n_pad) {
      atomicCAS(err, 0, 76);
      continue;
    }
    labels_m[(int64_t)b * n_pad + i] = sub[(int64_t)b * s_pad + j];
  }
}

static int row_grid(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  if (g > 64) g = 64;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace skcq

using namespace skcq;

extern "C" int skcq_mark_changed(const int32_t* prev, const int32_t* labels, int nblk, int n_pad, int k_pad,
                                 const int32_t* n, const int32_t* mask, int all, uint8_t* changed, void* stream) {
  SKCQ_REQUIRE(changed && n && (all || (prev && labels)), SKCQ_ERR_INVALID, "mark_changed: null pointer");
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535 && n_pad > 0 && k_pad > 0, SKCQ_ERR_INVALID, "mark_changed: bad sizes");
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "mark_changed: no device error word");
  cudaStream_t s = (cudaStream_t)stream;
  mark_reset_kernel<<<dim3(row_grid(k_pad, MC_THREADS), nblk), MC_THREADS, 0, s>>>(nblk, k_pad, mask, all, changed);
  if (!all)
    mark_diff_kernel<<<dim3(row_grid(n_pad, MC_THREADS), nblk), MC_THREADS, 0, s>>>(prev, labels, n_pad, k_pad, n,
                                                                                  mask, changed, err);
  return check_launch("mark_changed");
}

extern "C" size_t skcq_moved_lists_scratch_bytes(int nblk, int n_pad, int k_pad) {
  if (nblk <= 0 || n_pad <= 0 || k_pad <= 0) return 0;
  const int64_t chunks = ceil_div64(n_pad, CP_CHUNK) + ceil_div64(k_pad, CP_CHUNK);
  return (size_t)nblk * (size_t)chunks * sizeof(int32_t);
}

extern "C" int skcq_moved_lists(const uint8_t* changed, const int32_t* labels, int nblk, int n_pad, int k_pad,
                                const int32_t* n, const int32_t* k, const int32_t* mask, int32_t* mlist,
                                int32_t* mcount, int32_t* plist, int32_t* pcount, void* scratch,
                                size_t scratch_bytes, void* stream) {
  SKCQ_REQUIRE(changed && labels && n && k && mlist && mcount && plist && pcount && scratch, SKCQ_ERR_INVALID,
               "moved_lists: null pointer");
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535 && n_pad > 0 && k_pad > 0, SKCQ_ERR_INVALID, "moved_lists: bad sizes");
  SKCQ_REQUIRE(scratch_bytes >= skcq_moved_lists_scratch_bytes(nblk, n_pad, k_pad), SKCQ_ERR_INVALID,
               "moved_lists: scratch of %zu bytes, %zu needed", scratch_bytes,
               skcq_moved_lists_scratch_bytes(nblk, n_pad, k_pad));
  cudaStream_t s = (cudaStream_t)stream;
  const int kc = (int)ceil_div64(k_pad, CP_CHUNK), nc = (int)ceil_div64(n_pad, CP_CHUNK);
  int32_t* cnt_k = static_cast<int32_t*>(scratch);
  int32_t* cnt_n = cnt_k + (int64_t)nblk * kc;
  cp_count_kernel<<<dim3(kc, nblk), CP_THREADS, 0, s>>>(0, k_pad, n_pad, k_pad, n, k, mask, changed, labels, kc,
                                                         cnt_k);
  cp_place_kernel<<<dim3(kc, nblk), CP_THREADS, 0, s>>>(0, k_pad, n_pad, k_pad, n, k, mask, changed, labels, kc,
                                                         cnt_k, k_pad, mlist, mcount);
  cp_count_kernel<<<dim3(nc, nblk), CP_THREADS, 0, s>>>(1, n_pad, n_pad, k_pad, n, k, mask, changed, labels, nc,
                                                         cnt_n);
  cp_place_kernel<<<dim3(nc, nblk), CP_THREADS, 0, s>>>(1, n_pad, n_pad, k_pad, n, k, mask, changed, labels, nc,
                                                         cnt_n, n_pad, plist, pcount);
  return check_launch("moved_lists");
}

extern "C" int skcq_gather_rows(const float* src, int src_rows, const int32_t* idx, int idx_ld, const int32_t* count,
                                int nblk, int out_rows, int bs, float* dst, void* stream) {
  SKCQ_REQUIRE(src && idx && count && dst, SKCQ_ERR_INVALID, "gather_rows: null pointer");
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535 && src_rows > 0 && out_rows > 0 && bs > 0 && idx_ld >= out_rows,
               SKCQ_ERR_INVALID, "gather_rows: bad sizes");
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "gather_rows: no device error word");
  gather_rows_kernel<<<dim3(row_grid((int64_t)out_rows * bs, MC_THREADS), nblk), MC_THREADS, 0,
                       (cudaStream_t)stream>>>(src, src_rows, idx, idx_ld, count, out_rows, bs, dst, err);
  return check_launch("gather_rows");
}

extern "C" int skcq_assign_moved_exact(int metric, const float* X, const float* C, const float* cnorm, int nblk,
                                       int n_pad, int k_pad, int bs, const int32_t* n, const int32_t* active,
                                       const uint8_t* changed, const int32_t* mlist, const int32_t* mcount,
                                       int32_t* labels, const float* C_old, const float* cnorm_old, uint8_t* unres,
                                       void* stream) {
  SKCQ_REQUIRE(X && C && cnorm && n && changed && mlist && mcount && labels, SKCQ_ERR_INVALID,
               "assign_moved_exact: null pointer");
  SKCQ_REQUIRE(metric == SKCQ_METRIC_COSINE || metric == SKCQ_METRIC_L2, SKCQ_ERR_INVALID,
               "assign_moved_exact: metric");
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535 && n_pad > 0 && k_pad > 0 && bs > 0 && bs <= 32, SKCQ_ERR_INVALID,
               "assign_moved_exact: bad sizes (block size %d, at most 32)", bs);
  SKCQ_REQUIRE(!unres || (C_old && cnorm_old), SKCQ_ERR_INVALID, "assign_moved_exact: unres without old centroids");
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "assign_moved_exact: no device error word");
  const size_t smem = (size_t)MX_SLICE * (bs + 2) * sizeof(float);
  int64_t gx = (n_pad + MX_THREADS - 1) / MX_THREADS;
  const int64_t want = (148 * 8 + nblk - 1) / nblk;  // about 8 CTAs per SM over all problems
  if (gx > want) gx = want;
  dim3 grid((unsigned)(gx < 1 ? 1 : gx), (unsigned)nblk);
  cudaStream_t s = (cudaStream_t)stream;
#define SKCQ_MX(BSV)                                                                                           \
  assign_moved_exact_kernel<BSV><<<grid, MX_THREADS, smem, s>>>(metric, X, C, cnorm, n_pad, k_pad, bs, n, active, \
                                                                changed, mlist, mcount, labels, C_old, cnorm_old, \
                                                                unres, err)
  switch (bs) {
    case 4: SKCQ_MX(4); break;
    case 6: SKCQ_MX(6); break;
    case 8: SKCQ_MX(8); break;
    case 12: SKCQ_MX(12); break;
    case 16: SKCQ_MX(16); break;
    default: SKCQ_MX(0); break;
  }
#undef SKCQ_MX
  return check_launch("assign_moved_exact");
}

extern "C" int skcq_assign_merge(int metric, const float* X, const float* C, const float* cnorm, int nblk, int n_pad,
                                 int k_pad, int bs, const int32_t* n, const int32_t* active, const uint8_t* changed,
                                 const int32_t* mlist, const int32_t* mcount, const int32_t* labels_m,
                                 const int32_t* plist, const int32_t* pcount, int p_pad, const int32_t* labels_f,
                                 int32_t* labels, const float* C_old, const float* cnorm_old, uint8_t* unres,
                                 void* stream) {
  SKCQ_REQUIRE(X && C && cnorm && n && changed && mlist && mcount && labels_m && plist && pcount && labels &&
                   (p_pad == 0 || labels_f),
               SKCQ_ERR_INVALID, "assign_merge: null pointer");
  SKCQ_REQUIRE(!unres || (C_old && cnorm_old), SKCQ_ERR_INVALID, "assign_merge: unres without old centroids");
  SKCQ_REQUIRE(metric == SKCQ_METRIC_COSINE || metric == SKCQ_METRIC_L2, SKCQ_ERR_INVALID, "assign_merge: metric");
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535 && n_pad > 0 && k_pad > 0 && bs > 0 && p_pad >= 0 && p_pad <= n_pad,
               SKCQ_ERR_INVALID, "assign_merge: bad sizes");
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "assign_merge: no device error word");
  // phase 0 reads every point's previous label before phase 1 overwrites the
  // flagged ones
  for (int phase = 0; phase < 2; ++phase)
    assign_merge_kernel<<<dim3(row_grid(n_pad, MC_THREADS), nblk), MC_THREADS, 0, (cudaStream_t)stream>>>(
        metric, X, C, cnorm, n_pad, k_pad, bs, n, active, changed, mlist, mcount, labels_m, plist, pcount, p_pad,
        labels_f, labels, C_old, cnorm_old, unres, phase, err);
  return check_launch("assign_merge");
}

extern "C" int skcq_list_points(const uint8_t* flags, int nblk, int n_pad, const int32_t* n, const int32_t* mask,
                                int32_t* plist, int32_t* pcount, void* scratch, size_t scratch_bytes, void* stream) {
  SKCQ_REQUIRE(flags && n && plist && pcount && scratch, SKCQ_ERR_INVALID, "list_points: null pointer");
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535 && n_pad > 0, SKCQ_ERR_INVALID, "list_points: bad sizes");
  const int nc = (int)ceil_div64(n_pad, CP_CHUNK);
  SKCQ_REQUIRE(scratch_bytes >= (size_t)nblk * nc * sizeof(int32_t), SKCQ_ERR_INVALID,
               "list_points: scratch of %zu bytes", scratch_bytes);
  cudaStream_t s = (cudaStream_t)stream;
  int32_t* cnt = static_cast<int32_t*>(scratch);
  cp_count_kernel<<<dim3(nc, nblk), CP_THREADS, 0, s>>>(2, n_pad, n_pad, 1, n, n, mask, flags, nullptr, nc, cnt);
  cp_place_kernel<<<dim3(nc, nblk), CP_THREADS, 0, s>>>(2, n_pad, n_pad, 1, n, n, mask, flags, nullptr, nc, cnt,
                                                         n_pad, plist, pcount);
  return check_launch("list_points");
}

extern "C" int skcq_mpass_points(const float* X, const float* C, const int32_t* labels, const uint8_t* changed,
                                 const int32_t* n, const int32_t* active, int nblk, int n_pad, int k_pad, int bs,
                                 uint8_t* flags, void* stream) {
  SKCQ_REQUIRE(X && C && labels && changed && n && flags, SKCQ_ERR_INVALID, "mpass_points: null pointer");
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535 && n_pad > 0 && k_pad > 0 && bs > 0, SKCQ_ERR_INVALID,
               "mpass_points: bad sizes");
  mpass_points_kernel<<<dim3(row_grid(n_pad, MC_THREADS), nblk), MC_THREADS, 0, (cudaStream_t)stream>>>(
      X, C, labels, changed, n, active, n_pad, k_pad, bs, flags);
  return check_launch("mpass_points");
}

extern "C" int skcq_scatter_sub(const int32_t* list, const int32_t* count, const int32_t* sub, int nblk, int s_pad,
                                int n_pad, int32_t* labels_m, void* stream) {
  SKCQ_REQUIRE(list && count && sub && labels_m, SKCQ_ERR_INVALID, "scatter_sub: null pointer");
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535 && s_pad > 0 && n_pad >= s_pad, SKCQ_ERR_INVALID, "scatter_sub: bad sizes");
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "scatter_sub: no device error word");
  scatter_sub_kernel<<<dim3(row_grid(s_pad, MC_THREADS), nblk), MC_THREADS, 0, (cudaStream_t)stream>>>(
      list, count, sub, s_pad, n_pad, labels_m, err);
  return check_launch("scatter_sub");
}
