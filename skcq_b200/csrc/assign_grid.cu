// Exact nearest-centroid search for euclidean problems of block size 2-4
// through a grid over the centroids. No counterpart in the reference, whose
// assign_l2 scores every centroid (skcq/codebook/kmeans.py:46-66); the labels
// are the same: the arg-max of the reference formula (exact_score), first
// maximum, i.e. the labels skcq_assign_exact gives.
//
// Per problem:
//   1. bounds: per coordinate, G - 1 cell boundaries at quantiles of a sample
//      of the centroids (any non-decreasing boundaries give correct labels;
//      quantiles keep the cells' centroid counts even), and cmax >= max |c|
//      (NaN when a centroid coordinate is not finite: no point is certified).
//   2. count / scan / scatter: the centroids counting-sorted by fine cell
//      (coordinates, norms and indices in cell order), the points by
//      super-cell (GR_SUP fine cells per coordinate).
//   3. search: one warp per super-cell scores the super-cell's points against
//      every centroid of its fine cells and of one cell around them with the
//      reference formula, keeping the largest score (lowest index among
//      equals). A point is certified when no centroid outside that box can
//      win or tie: such a centroid c is at distance >= R from the point (R =
//      the point's distance to the box's nearest finite face), so its exact
//      value -2<x,c> + |c|^2 = |x - c|^2 - |x|^2 is >= R^2 - |x|^2, and its
//      fp32 value is within eps (2 |x| cmax + cmax^2) of the exact one (the
//      dot and the norm are fused multiply-add chains of bs terms, then two
//      roundings). When that lower bound (evaluated in double) is above the
//      winner's fp32 value, the winner is the arg-max over all centroids.
//      Uncertified points are flagged for a search over all centroids.
#include <math.h>

#include "common.cuh"

namespace skcq {

constexpr int GR_SUP = 2;          // fine cells per super-cell edge
constexpr int GR_SAMPLE = 4096;    // centroids sampled per problem for the boundaries
constexpr int GR_WARPS = 8;        // super-cells (one per warp) per CTA
constexpr int GR_CAPW = 256;       // candidates staged per warp and chunk
constexpr int GR_MAX_RUNS = 64;    // (GR_SUP + 2)^(bs - 1) runs of cells along coordinate 0
constexpr int GR_MAX_BND = 1024;   // bs * (G - 1) boundaries per problem
constexpr int GR_THREADS = 256;    // count / scatter kernels

struct GridScratch {
  float* bnd;        // [nblk][bs][G - 1]
  float* cmax;       // [nblk]
  int32_t* cpos;     // [nblk][ncell]: counts, exclusive starts, then (after the scatter) cell ends
  int32_t* ccell;    // [nblk][k_pad] fine cell of each centroid
  float4* csort;     // [nblk][k_pad] centroid coordinates in cell order (zero padded to 4)
  float* csn;        // [nblk][k_pad] their norms (cnorm)
  int32_t* cid;      // [nblk][k_pad] their indices
  int32_t* spos;     // [nblk][nsc] as cpos, per super-cell
  int32_t* pcell;    // [nblk][n_pad] super-cell of each point
  int32_t* porder;   // [nblk][n_pad] points in super-cell order
};

struct GridShape {
  int G, S;          // fine cells / super-cells per coordinate
  int64_t ncell;     // G^bs
  int nsc;           // S^bs
};

static GridShape grid_shape(int bs, int G) {
  GridShape g;
  g.G = G;
  g.S = (G + GR_SUP - 1) / GR_SUP;
  g.ncell = 1;
  int64_t nsc = 1;
  for (int d = 0; d < bs; ++d) {
    g.ncell *= G;
    nsc *= g.S;
  }
  g.nsc = (int)nsc;
  return g;
}

// Bytes of the scratch layout (base == nullptr) or the layout itself.
static size_t grid_layout(int nblk, int n_pad, int k_pad, int bs, const GridShape& g, char* base, GridScratch* s) {
  size_t off = 0;
  auto take = [&](size_t bytes) -> char* {
    char* p = base ? base + off : nullptr;
    off += (bytes + 255) & ~(size_t)255;
    return p;
  };
  const size_t nb = (size_t)nblk;
  char* p;
  p = take(nb * bs * (g.G - 1) * sizeof(float));
  if (s) s->bnd = reinterpret_cast<float*>(p);
  p = take(nb * sizeof(float));
  if (s) s->cmax = reinterpret_cast<float*>(p);
  p = take(nb * (size_t)g.ncell * sizeof(int32_t));
  if (s) s->cpos = reinterpret_cast<int32_t*>(p);
  p = take(nb * k_pad * sizeof(int32_t));
  if (s) s->ccell = reinterpret_cast<int32_t*>(p);
  p = take(nb * k_pad * sizeof(float4));
  if (s) s->csort = reinterpret_cast<float4*>(p);
  p = take(nb * k_pad * sizeof(float));
  if (s) s->csn = reinterpret_cast<float*>(p);
  p = take(nb * k_pad * sizeof(int32_t));
  if (s) s->cid = reinterpret_cast<int32_t*>(p);
  p = take(nb * (size_t)g.nsc * sizeof(int32_t));
  if (s) s->spos = reinterpret_cast<int32_t*>(p);
  p = take(nb * n_pad * sizeof(int32_t));
  if (s) s->pcell = reinterpret_cast<int32_t*>(p);
  p = take(nb * n_pad * sizeof(int32_t));
  if (s) s->porder = reinterpret_cast<int32_t*>(p);
  return off;
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Number of boundaries bd[0 .. nb) that are <= v (bd non-decreasing): the cell
// coordinate of v, in [0, nb]. A NaN v gets 0.
__device__ __forceinline__ int grid_coord(const float* bd, int nb, float v) {
  int lo = 0, hi = nb;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (bd[mid] <= v)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// 1. One CTA per problem.
__global__ void __launch_bounds__(1024) grid_bounds_kernel(const float* __restrict__ C, int k_pad, int bs, int G,
                                                           const int32_t* __restrict__ k,
                                                           const int32_t* __restrict__ active,
                                                           float* __restrict__ bnd, float* __restrict__ cmax) {
  __shared__ uint32_t s[GR_SAMPLE];
  __shared__ float red[32];
  const int b = blockIdx.x;
  if (active && !active[b]) return;
  const int kb = k[b];
  if (kb <= 0) return;
  const float* Cb = C + (int64_t)b * k_pad * bs;
  float mx = 0.f;
  int bad = 0;
  for (int c = threadIdx.x; c < kb; c += blockDim.x) {
    float q = 0.f;
    for (int j = 0; j < bs; ++j) {
      const float v = Cb[(int64_t)c * bs + j];
      bad |= !isfinite(v);
      q = __fmaf_rn(v, v, q);
    }
    mx = fmaxf(mx, q);
  }
  const int any_bad = __syncthreads_or(bad);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
    // sqrt of an fp32 sum of bs squares: a factor 1 + 1e-6 covers its
    // rounding, so cmax bounds every |c| from above
    cmax[b] = (any_bad || !isfinite(m)) ? NAN : sqrtf(m) * 1.000001f;
  }
  const int m = min(kb, GR_SAMPLE);
  int P = 1;
  while (P < m) P <<= 1;
  for (int d = 0; d < bs; ++d) {
    __syncthreads();
    for (int i = threadIdx.x; i < P; i += blockDim.x)
      s[i] = i < m ? float_key(Cb[((int64_t)i * kb / m) * bs + d]) : 0xffffffffu;
    __syncthreads();
    for (int kk = 2; kk <= P; kk <<= 1) {
      for (int j = kk >> 1; j > 0; j >>= 1) {
        for (int i = threadIdx.x; i < P; i += blockDim.x) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const uint32_t x = s[i], y = s[ixj];
            if ((x > y) == ((i & kk) == 0)) {
              s[i] = y;
              s[ixj] = x;
            }
          }
        }
        __syncthreads();
      }
    }
    for (int j = threadIdx.x; j < G - 1; j += blockDim.x)
      bnd[((int64_t)b * bs + d) * (G - 1) + j] = key_to_float(s[(int64_t)(j + 1) * m / G]);
  }
}

// 2a. Cell counts of centroids and super-cell counts of points.
__global__ void __launch_bounds__(GR_THREADS) grid_count_kernel(
    const float* __restrict__ X, const float* __restrict__ C, int n_pad, int k_pad, int bs, GridShape g,
    const int32_t* __restrict__ n, const int32_t* __restrict__ k, const int32_t* __restrict__ active,
    GridScratch sc) {
  __shared__ float sb[GR_MAX_BND];
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int nbd = g.G - 1;
  for (int t = threadIdx.x; t < bs * nbd; t += blockDim.x) sb[t] = sc.bnd[(int64_t)b * bs * nbd + t];
  __syncthreads();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int kb = k[b];
  if (i < kb) {
    const float* c = C + ((int64_t)b * k_pad + i) * bs;
    int cell = 0;
    for (int d = bs - 1; d >= 0; --d) cell = cell * g.G + grid_coord(sb + d * nbd, nbd, c[d]);
    sc.ccell[(int64_t)b * k_pad + i] = cell;
    atomicAdd(&sc.cpos[(int64_t)b * g.ncell + cell], 1);
  }
  if (kb > 0 && i < n[b]) {
    const float* x = X + ((int64_t)b * n_pad + i) * bs;
    int s = 0;
    for (int d = bs - 1; d >= 0; --d) s = s * g.S + grid_coord(sb + d * nbd, nbd, x[d]) / GR_SUP;
    sc.pcell[(int64_t)b * n_pad + i] = s;
    atomicAdd(&sc.spos[(int64_t)b * g.nsc + s], 1);
  }
}

// In-place exclusive scan of a[0 .. len) by one CTA.
__device__ void grid_scan(int32_t* a, int64_t len) {
  const int64_t per = (len + blockDim.x - 1) / blockDim.x;
  const int64_t lo = min(len, (int64_t)threadIdx.x * per), hi = min(len, lo + per);
  int s = 0;
  for (int64_t i = lo; i < hi; ++i) s += a[i];
  int tot;
  int run = block_exclusive_scan(s, &tot);
  for (int64_t i = lo; i < hi; ++i) {
    const int v = a[i];
    a[i] = run;
    run += v;
  }
  __syncthreads();
}

// 2b. One CTA per problem.
__global__ void __launch_bounds__(1024) grid_scan_kernel(GridShape g, const int32_t* __restrict__ active,
                                                         GridScratch sc) {
  const int b = blockIdx.x;
  if (active && !active[b]) return;
  grid_scan(sc.cpos + (int64_t)b * g.ncell, g.ncell);
  grid_scan(sc.spos + (int64_t)b * g.nsc, g.nsc);
}

// 2c. Centroids into cell order, points into super-cell order. Afterwards
// cpos[c] is the end of cell c (its start is cpos[c - 1], or 0).
__global__ void __launch_bounds__(GR_THREADS) grid_scatter_kernel(
    const float* __restrict__ C, const float* __restrict__ cnorm, int n_pad, int k_pad, int bs, GridShape g,
    const int32_t* __restrict__ n, const int32_t* __restrict__ k, const int32_t* __restrict__ active,
    GridScratch sc) {
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int kb = k[b];
  if (i < kb) {
    const int64_t ci = (int64_t)b * k_pad + i;
    const int slot = atomicAdd(&sc.cpos[(int64_t)b * g.ncell + sc.ccell[ci]], 1);
    const float* c = C + ci * bs;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int d = 0; d < bs; ++d) v[d] = c[d];
    const int64_t so = (int64_t)b * k_pad + slot;
    sc.csort[so] = make_float4(v[0], v[1], v[2], v[3]);
    sc.csn[so] = cnorm[ci];
    sc.cid[so] = i;
  }
  if (kb > 0 && i < n[b]) {
    const int64_t pi = (int64_t)b * n_pad + i;
    const int slot = atomicAdd(&sc.spos[(int64_t)b * g.nsc + sc.pcell[pi]], 1);
    sc.porder[(int64_t)b * n_pad + slot] = i;
  }
}

// Whether the winner (best, bid) over the centroids of the cell box
// [lo[d], hi[d]] is the winner over all centroids. A centroid c outside the
// box is at distance >= R (the point's distance to the box's nearest finite
// face) and at distance >= |c| - |x|, so its exact value
// -2<x,c> + |c|^2 = |x - c|^2 - |x|^2 is >= max(R, |c| - |x|)^2 - |x|^2, and
// its fp32 value is within eps (2 |x| |c| + |c|^2) of that (eps: 4x the
// score's rounding bound, (bs + 2) units of 2^-24). Over |c| this lower bound
// is smallest at |c| = rho = min(cmax, |x| + R) (for R >= 4 eps |x|; below
// that rho = cmax), so the winner is certified when
// R^2 - |x|^2 - eps (2 |x| rho + rho^2) exceeds its fp32 value -best.
// Evaluated in double with a margin for the double rounding. sb: the
// problem's boundaries, nbd = G - 1 per coordinate.
template <int BS>
__device__ __forceinline__ bool grid_certified(const float (&x)[BS], float best, int bid, const int (&lo)[BS],
                                               const int (&hi)[BS], const float* sb, int nbd, int G, float cm) {
  double xx = 0.0;
#pragma unroll
  for (int d = 0; d < BS; ++d) xx += (double)x[d] * (double)x[d];
  if (bid < 0 || !isfinite(best) || !isfinite(xx)) return false;
  double R = INFINITY;
#pragma unroll
  for (int d = 0; d < BS; ++d) {
    if (lo[d] > 0) R = fmin(R, (double)x[d] - (double)sb[d * nbd + lo[d] - 1]);
    if (hi[d] < G - 1) R = fmin(R, (double)sb[d * nbd + hi[d]] - (double)x[d]);
  }
  if (R == INFINITY) return true;  // the box is the whole grid
  const double eps = 4.0 * (BS + 2) * 5.9604644775390625e-08;
  const double nx = sqrt(xx), r2 = R * R;
  const double c = R >= 4.0 * eps * nx ? fmin((double)cm, nx + R) : (double)cm;
  const double lb = r2 - xx - eps * (2.0 * nx * c + c * c) - 1e-12 * (r2 + xx + fabs((double)best));
  return R >= 0.0 && lb > -(double)best;
}

// 3. One warp per super-cell, GR_WARPS super-cells of one problem per CTA.
struct GridSearchArgs {
  const float* X;
  int n_pad, k_pad;
  GridShape g;
  const int32_t* n;
  const int32_t* k;
  const int32_t* active;
  GridScratch sc;
  int32_t* labels;
  uint8_t* unres;
  int ring_max;  // largest box radius of the ring search (grid_ring_kernel)
};

constexpr size_t GR_SEARCH_SMEM =
    (size_t)GR_MAX_BND * sizeof(float) + (size_t)GR_WARPS * GR_CAPW * (sizeof(float4) + sizeof(float) + sizeof(int));

template <int BS>
__global__ void __launch_bounds__(GR_WARPS * 32) grid_search_kernel(GridSearchArgs a) {
  extern __shared__ __align__(16) unsigned char gsm[];
  float4* cand = reinterpret_cast<float4*>(gsm);                                   // [GR_WARPS][GR_CAPW]
  float* cnm = reinterpret_cast<float*>(gsm + (size_t)GR_WARPS * GR_CAPW * sizeof(float4));
  int* cidx = reinterpret_cast<int*>(cnm + GR_WARPS * GR_CAPW);
  float* sb = reinterpret_cast<float*>(cidx + GR_WARPS * GR_CAPW);                 // [BS][G - 1]
  __shared__ int run_start[GR_WARPS][GR_MAX_RUNS];
  __shared__ int run_off[GR_WARPS][GR_MAX_RUNS + 1];
  const int b = blockIdx.y;
  if (a.active && !a.active[b]) return;
  const int kb = a.k[b], np = a.n[b];
  if (kb <= 0 || np <= 0) return;
  const int G = a.g.G, S = a.g.S, nbd = G - 1;
  for (int t = threadIdx.x; t < BS * nbd; t += blockDim.x) sb[t] = a.sc.bnd[(int64_t)b * BS * nbd + t];
  __syncthreads();  // the only block-wide barrier; warps work alone from here
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int scell = blockIdx.x * GR_WARPS + warp;
  if (scell >= a.g.nsc) return;
  const int32_t* spos = a.sc.spos + (int64_t)b * a.g.nsc;
  const int p0 = scell ? spos[scell - 1] : 0, p1 = spos[scell];
  if (p0 >= p1) return;
  const int32_t* porder = a.sc.porder + (int64_t)b * a.n_pad;
  uint8_t* unres = a.unres + (int64_t)b * a.n_pad;
  const float cm = a.sc.cmax[b];
  if (!isfinite(cm)) {
    for (int p = p0 + lane; p < p1; p += 32) unres[porder[p]] = 1;
    return;
  }
  // the box: fine cells [lo[d], hi[d]] per coordinate
  int lo[BS], hi[BS];
  {
    int rem = scell;
#pragma unroll
    for (int d = 0; d < BS; ++d) {
      const int s = rem % S;
      rem /= S;
      lo[d] = max(0, s * GR_SUP - 1);
      hi[d] = min(G - 1, s * GR_SUP + GR_SUP);
    }
  }
  // runs of cells along coordinate 0 (contiguous in cell order)
  int nruns = 1;
#pragma unroll
  for (int d = 1; d < BS; ++d) nruns *= hi[d] - lo[d] + 1;
  const int32_t* cpos = a.sc.cpos + (int64_t)b * a.g.ncell;
  for (int r = lane; r < nruns; r += 32) {
    int rr = r;
    int64_t base = 0, mul = G;
#pragma unroll
    for (int d = 1; d < BS; ++d) {
      const int w = hi[d] - lo[d] + 1;
      base += (int64_t)(lo[d] + rr % w) * mul;
      rr /= w;
      mul *= G;
    }
    const int64_t c_lo = base + lo[0], c_hi = base + hi[0];
    const int st = c_lo ? cpos[c_lo - 1] : 0;
    run_start[warp][r] = st;
    run_off[warp][r + 1] = cpos[c_hi] - st;
  }
  __syncwarp();
  if (lane == 0) {
    int o = 0;
    for (int r = 0; r < nruns; ++r) {
      const int len = run_off[warp][r + 1];
      run_off[warp][r] = o;
      o += len;
    }
    run_off[warp][nruns] = o;
  }
  __syncwarp();
  const int total = run_off[warp][nruns];
  const int64_t cbase = (int64_t)b * a.k_pad;
  float4* wc = cand + warp * GR_CAPW;
  float* wn = cnm + warp * GR_CAPW;
  int* wi = cidx + warp * GR_CAPW;
  for (int pb = p0; pb < p1; pb += 32) {
    const int p = pb + lane;
    const bool live = p < p1;
    const int pi = live ? porder[p] : 0;
    float x[BS];
#pragma unroll
    for (int d = 0; d < BS; ++d) x[d] = live ? a.X[((int64_t)b * a.n_pad + pi) * BS + d] : 0.f;
    float best = -INFINITY;
    int bid = -1;
    for (int off = 0; off < total; off += GR_CAPW) {
      const int cnt = min(GR_CAPW, total - off);
      __syncwarp();
      for (int t = lane; t < cnt; t += 32) {
        const int gi = off + t;
        int l = 0, h = nruns - 1;  // the last run starting at or before gi
        while (l < h) {
          const int mid = (l + h + 1) >> 1;
          if (run_off[warp][mid] <= gi)
            l = mid;
          else
            h = mid - 1;
        }
        const int64_t src = cbase + run_start[warp][l] + (gi - run_off[warp][l]);
        wc[t] = a.sc.csort[src];
        wn[t] = a.sc.csn[src];
        wi[t] = a.sc.cid[src];
      }
      __syncwarp();
      if (live) {
        for (int t = 0; t < cnt; ++t) {
          const float4 cv = wc[t];
          const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
          float dot = 0.f;
#pragma unroll
          for (int d = 0; d < BS; ++d) dot = __fmaf_rn(x[d], cc[d], dot);
          const float s = -__fadd_rn(__fmul_rn(dot, -2.0f), wn[t]);  // exact_score, euclidean
          const int id = wi[t];
          if (s > best || (s == best && id < bid)) {
            best = s;
            bid = id;
          }
        }
      }
    }
    if (!live) continue;
    const bool ok = grid_certified<BS>(x, best, bid, lo, hi, sb, nbd, G, cm);
    if (ok) a.labels[(int64_t)b * a.n_pad + pi] = bid;
    unres[pi] = ok ? 0 : 1;
  }
}

// 4. Points the super-cell search left uncertified: one warp per point
// searches the box of fine cells [q - r, q + r] around the point's own cell q
// for r = GR_SUP .. ring_max (lanes split the box's runs of cells, then a
// warp reduction keeps the largest score, lowest index among equals) and
// stops at the first box it certifies. The rest stay flagged. Warps stride
// over the problem's points 32 at a time and take the flagged ones.
constexpr int GR_RING_MAX = 3;  // largest ring_max accepted

// Score one candidate with the reference formula (exact_score, euclidean) and
// keep it when it beats (best, bid): larger score, or equal with a lower index.
template <int BS>
__device__ __forceinline__ void grid_ring_take(const float (&x)[BS], float4 cv, float cn, int id, float& best,
                                               int& bid) {
  const float cc[4] = {cv.x, cv.y, cv.z, cv.w};
  float dot = 0.f;
#pragma unroll
  for (int d = 0; d < BS; ++d) dot = __fmaf_rn(x[d], cc[d], dot);
  const float s = -__fadd_rn(__fmul_rn(dot, -2.0f), cn);
  if (s > best || (s == best && id < bid)) {
    best = s;
    bid = id;
  }
}

template <int BS>
__global__ void __launch_bounds__(GR_WARPS * 32, 4) grid_ring_kernel(GridSearchArgs a) {
  __shared__ float sb[GR_MAX_BND];
  const int b = blockIdx.y;
  if (a.active && !a.active[b]) return;
  const int kb = a.k[b], np = a.n[b];
  if (kb <= 0 || np <= 0) return;
  const int G = a.g.G, nbd = G - 1;
  for (int t = threadIdx.x; t < BS * nbd; t += blockDim.x) sb[t] = a.sc.bnd[(int64_t)b * BS * nbd + t];
  __syncthreads();  // the only block-wide barrier
  const float cm = a.sc.cmax[b];
  if (!isfinite(cm)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* unres = a.unres + (int64_t)b * a.n_pad;
  const int32_t* cpos = a.sc.cpos + (int64_t)b * a.g.ncell;
  const int64_t cbase = (int64_t)b * a.k_pad;
  const int nchunks = (np + 31) / 32;
  for (int chunk = blockIdx.x * GR_WARPS + warp; chunk < nchunks; chunk += gridDim.x * GR_WARPS) {
    const int i0 = chunk * 32;
    uint32_t todo = __ballot_sync(0xffffffffu, i0 + lane < np && unres[i0 + lane] != 0);
    while (todo) {
      const int pi = i0 + __ffs(todo) - 1;
      todo &= todo - 1;
      float x[BS];
      int q[BS];
#pragma unroll
      for (int d = 0; d < BS; ++d) {
        x[d] = a.X[((int64_t)b * a.n_pad + pi) * BS + d];
        q[d] = grid_coord(sb + d * nbd, nbd, x[d]);
      }
      for (int r = GR_SUP; r <= a.ring_max; ++r) {
        int lo[BS], hi[BS];
        int nruns = 1;
#pragma unroll
        for (int d = 0; d < BS; ++d) {
          lo[d] = max(0, q[d] - r);
          hi[d] = min(G - 1, q[d] + r);
          if (d > 0) nruns *= hi[d] - lo[d] + 1;
        }
        float best = -INFINITY;
        int bid = -1;
        // lane l takes runs l, l + 32, ...: the bounds of four of them are
        // loaded together, then their candidates two at a time, so several
        // L2 reads are in flight per lane
        for (int run0 = lane; run0 < nruns; run0 += 4 * 32) {
          int st[4], en[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int run = run0 + 32 * u;
            st[u] = 0;
            en[u] = 0;
            if (run < nruns) {
              int rr = run;
              int64_t base = 0, mul = G;
#pragma unroll
              for (int d = 1; d < BS; ++d) {
                const int w = hi[d] - lo[d] + 1;
                base += (int64_t)(lo[d] + rr % w) * mul;
                rr /= w;
                mul *= G;
              }
              const int64_t c_lo = base + lo[0], c_hi = base + hi[0];
              st[u] = c_lo ? cpos[c_lo - 1] : 0;
              en[u] = cpos[c_hi];
            }
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            int t = st[u];
            for (; t + 1 < en[u]; t += 2) {
              const float4 c0 = a.sc.csort[cbase + t], c1 = a.sc.csort[cbase + t + 1];
              const float n0 = a.sc.csn[cbase + t], n1 = a.sc.csn[cbase + t + 1];
              const int i0 = a.sc.cid[cbase + t], i1 = a.sc.cid[cbase + t + 1];
              grid_ring_take<BS>(x, c0, n0, i0, best, bid);
              grid_ring_take<BS>(x, c1, n1, i1, best, bid);
            }
            if (t < en[u])
              grid_ring_take<BS>(x, a.sc.csort[cbase + t], a.sc.csn[cbase + t], a.sc.cid[cbase + t], best, bid);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ob = __shfl_xor_sync(0xffffffffu, best, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bid, o);
          if (oi >= 0 && (bid < 0 || ob > best || (ob == best && oi < bid))) {
            best = ob;
            bid = oi;
          }
        }
        if (grid_certified<BS>(x, best, bid, lo, hi, sb, nbd, G, cm)) {
          if (lane == 0) {
            a.labels[(int64_t)b * a.n_pad + pi] = bid;
            unres[pi] = 0;
          }
          break;
        }
      }
    }
  }
}

}  // namespace skcq

using namespace skcq;

static bool grid_args_ok(int bs, int G) {
  if (bs < 2 || bs > 4 || G < 2 || G > 256 || bs * (G - 1) > GR_MAX_BND) return false;
  const GridShape g = grid_shape(bs, G);
  return g.ncell <= (1 << 20) && g.nsc <= (1 << 20);
}

extern "C" size_t skcq_assign_grid_scratch_bytes(int nblk, int n_pad, int k_pad, int bs, int G) {
  if (nblk <= 0 || n_pad < 0 || k_pad < 0 || !grid_args_ok(bs, G)) return 0;
  return grid_layout(nblk, n_pad, k_pad, bs, grid_shape(bs, G), nullptr, nullptr);
}

extern "C" int skcq_assign_grid(const float* X, const float* C, const float* cnorm, int nblk, int n_pad, int k_pad,
                                int bs, const int32_t* n, const int32_t* k, const int32_t* active, int G,
                                int ring_max, int32_t* labels, uint8_t* unres, void* scratch, size_t scratch_bytes,
                                void* stream) {
  SKCQ_REQUIRE(X && C && cnorm && n && k && labels && unres && scratch, SKCQ_ERR_INVALID,
               "assign_grid: null pointer");
  SKCQ_REQUIRE(grid_args_ok(bs, G), SKCQ_ERR_INVALID, "assign_grid: block size %d / %d cells per coordinate", bs, G);
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535 && n_pad >= 0 && k_pad >= 0, SKCQ_ERR_INVALID,
               "assign_grid: %d problems, n_pad %d, k_pad %d", nblk, n_pad, k_pad);
  SKCQ_REQUIRE(((uintptr_t)scratch & 255) == 0, SKCQ_ERR_INVALID, "assign_grid: scratch not 256-byte aligned");
  SKCQ_REQUIRE(ring_max == 0 || (ring_max >= GR_SUP && ring_max <= GR_RING_MAX), SKCQ_ERR_INVALID,
               "assign_grid: ring radius %d outside {0, %d .. %d}", ring_max, GR_SUP, GR_RING_MAX);
  const GridShape g = grid_shape(bs, G);
  GridScratch sc;
  const size_t need = grid_layout(nblk, n_pad, k_pad, bs, g, static_cast<char*>(scratch), &sc);
  SKCQ_REQUIRE(scratch_bytes >= need, SKCQ_ERR_INVALID, "assign_grid: scratch %zu bytes, need %zu", scratch_bytes,
               need);
  if (n_pad == 0 || k_pad == 0) return SKCQ_OK;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(sc.cpos, 0, (size_t)nblk * g.ncell * sizeof(int32_t), s);
  if (e == cudaSuccess) e = cudaMemsetAsync(sc.spos, 0, (size_t)nblk * g.nsc * sizeof(int32_t), s);
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "assign_grid: %s", cudaGetErrorString(e));
  grid_bounds_kernel<<<nblk, 1024, 0, s>>>(C, k_pad, bs, G, k, active, sc.bnd, sc.cmax);
  const dim3 pgrid(ceil_div(max(n_pad, k_pad), GR_THREADS), nblk);
  grid_count_kernel<<<pgrid, GR_THREADS, 0, s>>>(X, C, n_pad, k_pad, bs, g, n, k, active, sc);
  grid_scan_kernel<<<nblk, 1024, 0, s>>>(g, active, sc);
  grid_scatter_kernel<<<pgrid, GR_THREADS, 0, s>>>(C, cnorm, n_pad, k_pad, bs, g, n, k, active, sc);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    for (auto fn : {grid_search_kernel<2>, grid_search_kernel<3>, grid_search_kernel<4>}) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GR_SEARCH_SMEM);
      if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "assign_grid: %s", cudaGetErrorString(e));
    }
    configured_dev = dev;
  }
  GridSearchArgs args{X, n_pad, k_pad, g, n, k, active, sc, labels, unres, ring_max};
  const dim3 sgrid(ceil_div(g.nsc, GR_WARPS), nblk);
  const dim3 rgrid(min(ceil_div(ceil_div(n_pad, 32), GR_WARPS), 64), nblk);
  switch (bs) {
    case 2:
      grid_search_kernel<2><<<sgrid, GR_WARPS * 32, GR_SEARCH_SMEM, s>>>(args);
      if (ring_max) grid_ring_kernel<2><<<rgrid, GR_WARPS * 32, 0, s>>>(args);
      break;
    case 3:
      grid_search_kernel<3><<<sgrid, GR_WARPS * 32, GR_SEARCH_SMEM, s>>>(args);
      if (ring_max) grid_ring_kernel<3><<<rgrid, GR_WARPS * 32, 0, s>>>(args);
      break;
    default:
      grid_search_kernel<4><<<sgrid, GR_WARPS * 32, GR_SEARCH_SMEM, s>>>(args);
      if (ring_max) grid_ring_kernel<4><<<rgrid, GR_WARPS * 32, 0, s>>>(args);
      break;
  }
  return check_launch("assign_grid");
}
