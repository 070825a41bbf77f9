// Exact fp32 nearest-centroid assignment on CUDA cores: every score is the
// reference formula (skcq/codebook/kmeans.py:41-42, 63-65) evaluated in fp32.
// Cross-check for the tensor-core kernel; O(n * K * bs) FMAs.
#include "common.cuh"

namespace skcq {

constexpr int EXACT_THREADS = 256;
constexpr int EXACT_TILE = 256;  // centroids staged in shared memory per step

__global__ void __launch_bounds__(EXACT_THREADS)
assign_exact_kernel(int metric, const float* __restrict__ X, const float* __restrict__ C,
                    const float* __restrict__ cnorm, int n_pad, int k_pad, int bs, const int32_t* __restrict__ n,
                    const int32_t* __restrict__ k, const int32_t* __restrict__ active, int32_t* __restrict__ labels) {
  extern __shared__ float sm[];
  float* sc = sm;                        // [EXACT_TILE][bs]
  float* sn = sm + EXACT_TILE * bs;      // [EXACT_TILE]
  const int b = blockIdx.y;
  if (active && !active[b]) return;
  const int nb = n[b], kb = k[b];
  const int i = blockIdx.x * EXACT_THREADS + threadIdx.x;
  if (blockIdx.x * EXACT_THREADS >= nb) return;
  float x[64];
  if (i < nb)
    for (int j = 0; j < bs; ++j) x[j] = X[((int64_t)b * n_pad + i) * bs + j];
  float best = -INFINITY;
  int bi = 0;
  const float* Cb = C + (int64_t)b * k_pad * bs;
  for (int c0 = 0; c0 < kb; c0 += EXACT_TILE) {
    const int cnt = min(EXACT_TILE, kb - c0);
    __syncthreads();
    for (int t = threadIdx.x; t < cnt * bs; t += EXACT_THREADS) sc[t] = Cb[(int64_t)c0 * bs + t];
    for (int t = threadIdx.x; t < cnt; t += EXACT_THREADS) sn[t] = cnorm[(int64_t)b * k_pad + c0 + t];
    __syncthreads();
    if (i < nb) {
      for (int c = 0; c < cnt; ++c) {
        float s = exact_score(metric, x, sc + c * bs, sn[c], bs);
        if (s > best) {
          best = s;
          bi = c0 + c;
        }
      }
    }
  }
  if (i < nb) labels[(int64_t)b * n_pad + i] = bi;
}

}  // namespace skcq

using namespace skcq;

extern "C" int skcq_assign_exact(int metric, const float* X, const float* C, const float* cnorm, int nblk, int n_pad,
                                 int k_pad, int bs, const int32_t* n, const int32_t* k, const int32_t* active,
                                 int32_t* labels, void* stream) {
  SKCQ_REQUIRE(X && C && cnorm && n && k && labels, SKCQ_ERR_INVALID, "assign_exact: null pointer");
  SKCQ_REQUIRE(bs > 0 && bs <= 64, SKCQ_ERR_INVALID, "assign_exact: block size %d outside [1, 64]", bs);
  SKCQ_REQUIRE(nblk > 0 && nblk <= 65535, SKCQ_ERR_INVALID, "assign_exact: %d problems exceed 65535", nblk);
  dim3 grid(ceil_div(n_pad, EXACT_THREADS), nblk);
  size_t smem = (size_t)EXACT_TILE * (bs + 1) * sizeof(float);
  assign_exact_kernel<<<grid, EXACT_THREADS, smem, (cudaStream_t)stream>>>(metric, X, C, cnorm, n_pad, k_pad, bs, n,
                                                                           k, active, labels);
  return check_launch("assign_exact");
}
