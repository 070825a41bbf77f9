// Prefill forward of the codebook experts on the 5th-generation tensor cores
// (skcq/codebook_experts.py:30-61 gather_matmul mode, batched over experts).
//
// For large batches every active expert's weight is needed by many rows, so
// the weight is decoded once per forward instead of once per row:
//   1. plan:    128-row tiles of each expert's run of sorted (token, slot) rows;
//   2. pack:    the rows, gathered by token (or SwiGLU of gate/up), as bf16 in
//               the tcgen05 no-swizzle K-major shared-memory image, one
//               16 KB chunk (128 rows x 64 k) after another;
//   3. dequant: each active expert's W[out][in] = sum over codebooks of
//               scale * sign * C_b[idx] (+ raw remainder columns), bf16, in the
//               same image layout, 32 KB chunks of 256 outputs x 64 k;
//   4. gemm:    persistent CTAs walk (row tile, 256-output tile) items: a
//               producer warp streams A and B chunks with 1-D bulk copies into
//               a 4-stage ring, one thread issues tcgen05.mma kind::f16
//               (M=128, N=256, K=16 per instruction) into one of two TMEM
//               accumulators, four warps read it back with tcgen05.ld and
//               store fp32 rows (or SwiGLU rows for the next GEMM) while the
//               next item accumulates in the other.
// Because the packer and the decoder write the exact shared-memory image, no
// tensor map is needed: each stage is two contiguous bulk copies.
#include <cuda_bf16.h>

#include <algorithm>

#include "common.cuh"
#include "fwd_common.cuh"

namespace skcq {

constexpr int PF_BM = 128;
constexpr int PF_BN = 256;
constexpr int PF_BK = 64;
constexpr int PF_STAGES = 4;
constexpr uint32_t PF_A_BYTES = PF_BM * PF_BK * 2;  // 16 KB
constexpr uint32_t PF_B_BYTES = PF_BN * PF_BK * 2;  // 32 KB
constexpr int PF_THREADS = 192;                     // producer, MMA, 4 epilogue warps
constexpr size_t PF_SMEM = (size_t)PF_STAGES * (PF_A_BYTES + PF_B_BYTES) + 2048;  // + alignment pad and barriers

// Instruction descriptor: kind::f16 with bf16 A and B (K-major), f32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16-byte unit index of (row r, k-group kg) in a rows x 64 chunk: core matrices
// of 8 rows x 8 bf16, K-adjacent ones 128 B apart, 8-row groups 1 KB apart.
__device__ __forceinline__ int canon_unit(int r, int kg) { return ((r >> 3) * 8 + kg) * 8 + (r & 7); }

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// ---------------------------------------------------------------------------
// 1. plan: tiles[0] = n_tiles; tile t at tiles[1 + 3t ..]: (row0, row1, slot)
// ---------------------------------------------------------------------------
__global__ void prefill_plan_kernel(const int32_t* __restrict__ seg, int E, int max_tiles, int32_t* __restrict__ tiles,
                                    int* err) {
  __shared__ int s_base, s_sbase;
  if (threadIdx.x == 0) {
    s_base = 0;
    s_sbase = 0;
  }
  __syncthreads();
  for (int e0 = 0; e0 < E; e0 += 1024) {
    const int e = e0 + threadIdx.x;
    const int cnt = e < E ? seg[e + 1] - seg[e] : 0;
    int tot, stot;
    const int nt = (cnt + PF_BM - 1) / PF_BM;
    const int off = block_exclusive_scan(nt, &tot);
    const int soff = block_exclusive_scan(cnt > 0 ? 1 : 0, &stot);
    const int base = s_base + off, sbase = s_sbase + soff;
    if (e < E) {
      for (int t = 0; t < nt; ++t) {
        const int id = base + t;
        if (id >= max_tiles) {
          atomicCAS(err, 0, 44);
          break;
        }
        tiles[1 + 3 * id] = seg[e] + t * PF_BM;
        tiles[2 + 3 * id] = min(seg[e] + (t + 1) * PF_BM, seg[e + 1]);
        tiles[3 + 3 * id] = sbase;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      s_base += tot;
      s_sbase += stot;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) tiles[0] = min(s_base, max_tiles);
}

// ---------------------------------------------------------------------------
// 2. pack rows: A[t][kc] chunks (128 x 64 bf16 image)
// mode 0: row r reads x[row_token[r] % T] (f32 | bf16); mode 1: silu(g[r]) * u[r]
// ---------------------------------------------------------------------------
__global__ void prefill_pack_kernel(int mode, const void* __restrict__ x, int x_dtype, int64_t x_ld,
                                    const int32_t* __restrict__ row_token, int T, const float* __restrict__ u,
                                    int64_t u_ld, int in_dim, int KC, const int32_t* __restrict__ tiles,
                                    int max_tiles, uint4* __restrict__ A) {
  const int n_tiles = tiles[0];
  const int64_t units = (int64_t)max_tiles * KC * 1024;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < units; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / ((int64_t)KC * 1024));
    if (t >= n_tiles) break;  // tiles are outermost: the rest of this thread's units are past n_tiles too
    const int rem = (int)(i - (int64_t)t * KC * 1024);
    const int kc = rem >> 10, unit = rem & 1023;
    const int rg = unit >> 6, kg = (unit >> 3) & 7, r = rg * 8 + (unit & 7);
    const int row = tiles[1 + 3 * t] + r, row1 = tiles[2 + 3 * t];
    const int k0 = kc * PF_BK + kg * 8;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = 0.f;
    if (row < row1) {
      if (mode == 0) {
        const int64_t tok = row_token ? (int64_t)(row_token[row] % T) : (int64_t)row;
        if (x_dtype == SKCQ_DTYPE_BF16) {
          const uint16_t* p = static_cast<const uint16_t*>(x) + tok * x_ld + k0;
          if (k0 + 8 <= in_dim && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
            const uint4 q = *reinterpret_cast<const uint4*>(p);
            A[i] = q;
            continue;
          }
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (k0 + j < in_dim) v[j] = __uint_as_float((uint32_t)p[j] << 16);
        } else {
          const float* p = static_cast<const float*>(x) + tok * x_ld + k0;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (k0 + j < in_dim) v[j] = p[j];
        }
      } else {
        const float* g = static_cast<const float*>(x) + (int64_t)row * x_ld + k0;
        const float* uu = u + (int64_t)row * u_ld + k0;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (k0 + j < in_dim) {
            const float a = g[j];
            v[j] = __fdiv_rn(a, 1.0f + expf(-a)) * uu[j];
          }
      }
    }
    A[i] = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                      pack_bf16x2(v[6], v[7]));
  }
}

// ---------------------------------------------------------------------------
// 3. dequant: W[slot][nt][kc] chunks (256 x 64 bf16 image) of active experts
// ---------------------------------------------------------------------------
struct DqSet {
  skcq_fwd_layer l[SKCQ_MAX_CODECS];
  int n;
};

// One CTA per 32 KB chunk of W (256 image rows x 64 columns) of one expert;
// thread rr owns image row rr and accumulates its 64 columns in a private
// shared-memory row (stride 65 floats: conflict-free), adding for every layer
// the scaled, signed centroid of each block that overlaps the chunk (and raw
// remainder columns), then writes its eight 16-byte units. blockIdx.y (the
// chunk's column range) varies slowest, so the CTAs in flight read the same
// blocks' centroid tables and those stay in L2.
constexpr int DQ_THREADS = 256;
constexpr int DQ_LD = PF_BK + 1;

template <int BS, typename T>
__device__ __forceinline__ void dq_blocks(const skcq_fwd_layer& L, bool scaled, int e, int o, int out, int c0,
                                          float* __restrict__ acc) {
  const int nb = L.n_blocks;
  const int b_lo = c0 / BS;
  const int b_hi = min(nb, (c0 + PF_BK + BS - 1) / BS);
  const T* table = static_cast<const T*>(L.table);
  const uint16_t* ix = L.idx16 + (int64_t)e * nb * out + o;
  const uint32_t* sg = L.sign_mask ? L.sign_mask + (int64_t)e * nb * out + o : nullptr;
  constexpr int U = BS <= 4 ? 8 : 4;
  int b = b_lo;
  for (; b + U <= b_hi; b += U) {
    int idx[U];
#pragma unroll
    for (int u = 0; u < U; ++u) idx[u] = __ldg(ix + (int64_t)(b + u) * out);
    float w[U][BS];
#pragma unroll
    for (int u = 0; u < U; ++u) load_centroid<BS, T>(table + ((int64_t)(b + u) * L.K + idx[u]) * BS, w[u]);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t eb = ((int64_t)e * nb + b + u) * out + o;
      const uint32_t m = sg ? __ldg(sg + (int64_t)(b + u) * out) : 0u;
      const float sc = scaled ? ld_scale(L.scales, eb, L.scale_dtype, L.q_scale) : 1.f;
      const int col0 = (b + u) * BS - c0;
#pragma unroll
      for (int j = 0; j < BS; ++j) {
        const int col = col0 + j;
        if (col >= 0 && col < PF_BK) {
          const float v = (m >> j & 1u) ? -w[u][j] : w[u][j];
          acc[col] = scaled ? __fmaf_rn(v, sc, acc[col]) : acc[col] + v;
        }
      }
    }
  }
  for (; b < b_hi; ++b) {
    const int idx = __ldg(ix + (int64_t)b * out);
    float w[BS];
    load_centroid<BS, T>(table + ((int64_t)b * L.K + idx) * BS, w);
    const int64_t eb = ((int64_t)e * nb + b) * out + o;
    const uint32_t m = sg ? __ldg(sg + (int64_t)b * out) : 0u;
    const float sc = scaled ? ld_scale(L.scales, eb, L.scale_dtype, L.q_scale) : 1.f;
#pragma unroll
    for (int j = 0; j < BS; ++j) {
      const int col = b * BS + j - c0;
      if (col >= 0 && col < PF_BK) {
        const float v = (m >> j & 1u) ? -w[j] : w[j];
        acc[col] = scaled ? __fmaf_rn(v, sc, acc[col]) : acc[col] + v;
      }
    }
  }
}

// any block size <= 32: element loads
template <typename T>
__device__ __forceinline__ void dq_blocks_any(const skcq_fwd_layer& L, bool scaled, int e, int o, int out, int c0,
                                              float* __restrict__ acc) {
  const int nb = L.n_blocks, bs = L.bs;
  const T* table = static_cast<const T*>(L.table);
  const int b_lo = c0 / bs, b_hi = min(nb, (c0 + PF_BK + bs - 1) / bs);
  for (int b = b_lo; b < b_hi; ++b) {
    const int64_t eb = ((int64_t)e * nb + b) * out + o;
    const int idx = L.idx16[eb];
    const uint32_t m = L.sign_mask ? L.sign_mask[eb] : 0u;
    const float sc = scaled ? ld_scale(L.scales, eb, L.scale_dtype, L.q_scale) : 1.f;
    for (int j = 0; j < bs; ++j) {
      const int col = b * bs + j - c0;
      if (col < 0 || col >= PF_BK) continue;
      float v;
      if constexpr (sizeof(T) == 4)
        v = reinterpret_cast<const float*>(table)[((int64_t)b * L.K + idx) * bs + j];
      else
        v = __uint_as_float((uint32_t) reinterpret_cast<const uint16_t*>(table)[((int64_t)b * L.K + idx) * bs + j]
                            << 16);
      if (m >> j & 1u) v = -v;
      acc[col] = scaled ? __fmaf_rn(v, sc, acc[col]) : acc[col] + v;
    }
  }
}

template <typename T>
__device__ __forceinline__ void dq_layer(const skcq_fwd_layer& L, bool scaled, int e, int o, int out, int c0,
                                         float* acc) {
  switch (L.bs) {
    case 4: dq_blocks<4, T>(L, scaled, e, o, out, c0, acc); break;
    case 6: dq_blocks<6, T>(L, scaled, e, o, out, c0, acc); break;
    case 8: dq_blocks<8, T>(L, scaled, e, o, out, c0, acc); break;
    case 12: dq_blocks<12, T>(L, scaled, e, o, out, c0, acc); break;
    case 16: dq_blocks<16, T>(L, scaled, e, o, out, c0, acc); break;
    default: dq_blocks_any<T>(L, scaled, e, o, out, c0, acc); break;
  }
  // raw remainder columns [cov, cov + rem) (codebook_experts.py:64-74)
  const int cov = L.n_blocks * L.bs;
  const int lo = max(cov, c0), hi = min(cov + L.rem, c0 + PF_BK);
  for (int c = lo; c < hi; ++c) acc[c - c0] += ld_any(L.remainder, ((int64_t)e * out + o) * L.rem + (c - cov), L.rem_dtype);
}

// half < 0: image rows are 256 outputs; half = 0 | 1: image rows [128 half,
// 128 half + 128) hold this module's 128 features (gate and up interleaved).
__global__ void __launch_bounds__(DQ_THREADS, 3) prefill_dequant_kernel(DqSet set, const int32_t* __restrict__ active,
                                                                     int out, int in_dim, int NT, int KC, int half,
                                                                     uint4* __restrict__ W) {
  extern __shared__ float dq_acc[];  // [DQ_THREADS][DQ_LD]
  const int n_slots = active ? active[0] : (int)(gridDim.x / NT);
  const int slot = blockIdx.x / NT, nt = blockIdx.x - slot * NT, kc = blockIdx.y;
  if (slot >= n_slots) return;
  const int e = active ? active[1 + slot] : slot;
  // half < 0: 256 threads, one per image row; half >= 0: 128 threads for this
  // module's rows [128 half, 128 half + 128)
  const int rr = threadIdx.x + (half < 0 ? 0 : half * (PF_BN / 2));
  const int o = half < 0 ? nt * PF_BN + rr : nt * (PF_BN / 2) + threadIdx.x;
  if (o >= out) return;  // rows past out_dim stay unwritten: their accumulator columns are never stored
  float* acc = dq_acc + threadIdx.x * DQ_LD;
#pragma unroll 8
  for (int c = 0; c < PF_BK; ++c) acc[c] = 0.f;
  const int c0 = kc * PF_BK;
  if (c0 < in_dim) {
    for (int li = 0; li < set.n; ++li) {
      const skcq_fwd_layer& L = set.l[li];
      const bool scaled = li == 0 && L.scales != nullptr;
      if (L.table_dtype == SKCQ_DTYPE_BF16)
        dq_layer<__nv_bfloat16>(L, scaled, e, o, out, c0, acc);
      else
        dq_layer<float>(L, scaled, e, o, out, c0, acc);
    }
    for (int c = max(0, in_dim - c0); c < PF_BK; ++c) acc[c] = 0.f;  // K padding
  }
  uint4* chunk = W + (((int64_t)slot * NT + nt) * KC + kc) * (PF_B_BYTES / 16);
#pragma unroll
  for (int kg = 0; kg < 8; ++kg) {
    const float* a = acc + kg * 8;
    chunk[canon_unit(rr, kg)] = make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]),
                                           pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
  }
}

// Fast path for bf16 tables and up to three layers whose block sizes divide
// a 32-column strip (4, 8 or 16; 0 = no such layer): the strip's columns are
// accumulated in registers at compile-time positions, and each layer's index
// loads are issued before its centroid gathers (8 at a time), so a thread
// keeps a layer's loads in flight and touches no shared memory.
template <int BS, int CW>
__device__ __forceinline__ void dqf_layer(const skcq_fwd_layer& L, bool scaled, int e, int o, int out, int c0,
                                          float (&acc)[CW]) {
  if constexpr (BS > 0) {
    constexpr int NBC = CW / BS;
    const int nb = L.n_blocks;
    const int b0 = c0 / BS;
    const __nv_bfloat16* table = static_cast<const __nv_bfloat16*>(L.table);
    const uint16_t* ix = L.idx16 + (int64_t)e * nb * out + o;
    const int cov = nb * BS;
    // blocks per batch of loads: at most 16 gathered values in flight per
    // thread, which keeps the strip's accumulators in registers
    constexpr int G = (16 / BS) < NBC ? (16 / BS > 0 ? 16 / BS : 1) : NBC;
#pragma unroll
    for (int g0 = 0; g0 < NBC; g0 += G) {
    int idx[G];
#pragma unroll
    for (int u = 0; u < G; ++u) idx[u] = (b0 + g0 + u < nb) ? (int)__ldg(ix + (int64_t)(b0 + g0 + u) * out) : 0;
#pragma unroll
    for (int uu = 0; uu < G; ++uu) {
      const int u = g0 + uu;
      const int b = b0 + u;
      if (b < nb) {
        float w[BS];
        load_centroid<BS, __nv_bfloat16>(table + ((int64_t)b * L.K + idx[uu]) * BS, w);
        const int64_t eb = ((int64_t)e * nb + b) * out + o;
        const uint32_t m = L.sign_mask ? __ldg(L.sign_mask + eb) : 0u;
        const float sc = scaled ? ld_scale(L.scales, eb, L.scale_dtype, L.q_scale) : 1.f;
#pragma unroll
        for (int j = 0; j < BS; ++j) {
          const float v = (m >> j & 1u) ? -w[j] : w[j];
          acc[u * BS + j] = scaled ? __fmaf_rn(v, sc, acc[u * BS + j]) : acc[u * BS + j] + v;
        }
      } else if (L.rem > 0) {
        // raw remainder columns [cov, cov + rem) (codebook_experts.py:64-74)
#pragma unroll
        for (int j = 0; j < BS; ++j) {
          const int col = b * BS + j - cov;
          if (col >= 0 && col < L.rem)
            acc[u * BS + j] += ld_any(L.remainder, ((int64_t)e * out + o) * L.rem + col, L.rem_dtype);
        }
      }
    }
    }
  }
}

// Two threads per image row, each owning 32 of the chunk's 64 columns (half
// the accumulator registers of one thread per row, so twice the warps fit).
constexpr int DQF_CW = PF_BK / 2;

template <int BS0, int BS1, int BS2>
__global__ void __launch_bounds__(2 * DQ_THREADS, 2) prefill_dequant_fast_kernel(DqSet set,
                                                                                const int32_t* __restrict__ active,
                                                                                int out, int in_dim, int NT, int KC,
                                                                                int half, uint4* __restrict__ W) {
  const int n_slots = active ? active[0] : (int)(gridDim.x / NT);
  const int slot = blockIdx.x / NT, nt = blockIdx.x - slot * NT, kc = blockIdx.y;
  if (slot >= n_slots) return;
  const int e = active ? active[1 + slot] : slot;
  const int rows = blockDim.x >> 1;  // image rows of this launch (256, or 128 per interleaved module)
  const int strip = threadIdx.x / rows, tr = threadIdx.x - strip * rows;
  const int rr = tr + (half < 0 ? 0 : half * (PF_BN / 2));
  const int o = half < 0 ? nt * PF_BN + rr : nt * (PF_BN / 2) + tr;
  if (o >= out) return;  // rows past out_dim stay unwritten: their accumulator columns are never stored
  float acc[DQF_CW];
#pragma unroll
  for (int c = 0; c < DQF_CW; ++c) acc[c] = 0.f;
  const int c0 = kc * PF_BK + strip * DQF_CW;
  if (c0 < in_dim) {
    dqf_layer<BS0, DQF_CW>(set.l[0], set.l[0].scales != nullptr, e, o, out, c0, acc);
    if (set.n > 1) dqf_layer<BS1, DQF_CW>(set.l[1], false, e, o, out, c0, acc);
    if (set.n > 2) dqf_layer<BS2, DQF_CW>(set.l[2], false, e, o, out, c0, acc);
#pragma unroll
    for (int c = 0; c < DQF_CW; ++c)
      if (c0 + c >= in_dim) acc[c] = 0.f;  // K padding
  }
  uint4* chunk = W + (((int64_t)slot * NT + nt) * KC + kc) * (PF_B_BYTES / 16);
#pragma unroll
  for (int q = 0; q < DQF_CW / 8; ++q)
    chunk[canon_unit(rr, strip * (DQF_CW / 8) + q)] =
        make_uint4(pack_bf16x2(acc[q * 8], acc[q * 8 + 1]), pack_bf16x2(acc[q * 8 + 2], acc[q * 8 + 3]),
                   pack_bf16x2(acc[q * 8 + 4], acc[q * 8 + 5]), pack_bf16x2(acc[q * 8 + 6], acc[q * 8 + 7]));
}

using DqFastFn = void (*)(DqSet, const int32_t*, int, int, int, int, int, uint4*);

template <int BS0, int BS1>
DqFastFn dq_fast_pick3(int bs2) {
  switch (bs2) {
    case 0: return prefill_dequant_fast_kernel<BS0, BS1, 0>;
    case 4: return prefill_dequant_fast_kernel<BS0, BS1, 4>;
    case 8: return prefill_dequant_fast_kernel<BS0, BS1, 8>;
    case 16: return prefill_dequant_fast_kernel<BS0, BS1, 16>;
    default: return nullptr;
  }
}

template <int BS0>
DqFastFn dq_fast_pick2(int bs1, int bs2) {
  switch (bs1) {
    case 0: return bs2 == 0 ? prefill_dequant_fast_kernel<BS0, 0, 0> : nullptr;
    case 4: return dq_fast_pick3<BS0, 4>(bs2);
    case 8: return dq_fast_pick3<BS0, 8>(bs2);
    case 16: return dq_fast_pick3<BS0, 16>(bs2);
    default: return nullptr;
  }
}

// The fast-path instantiation for these layers, or nullptr.
inline DqFastFn dq_fast_pick(const DqSet& set) {
  if (set.n > 3) return nullptr;
  int bs[3] = {0, 0, 0};
  for (int i = 0; i < set.n; ++i) {
    if (set.l[i].table_dtype != SKCQ_DTYPE_BF16) return nullptr;
    bs[i] = set.l[i].bs;
  }
  switch (bs[0]) {
    case 4: return dq_fast_pick2<4>(bs[1], bs[2]);
    case 8: return dq_fast_pick2<8>(bs[1], bs[2]);
    case 16: return dq_fast_pick2<16>(bs[1], bs[2]);
    default: return nullptr;
  }
}

// ---------------------------------------------------------------------------
// 4. grouped GEMM on tcgen05
// ---------------------------------------------------------------------------
struct GemmArgs {
  const uint8_t* A;  // [max_tiles][KC] 16 KB chunks
  const uint8_t* W;  // [slots][NT][KC] 32 KB chunks
  const int32_t* tiles;
  int KC, NT, out;
  void* y;  // mode 0: rows, f32 or bf16 (y_dtype)
  int y_dtype;
  int64_t y_ld;
  uint4* a_out;  // mode 1: SwiGLU rows in the A image ([max_tiles][KC_out] chunks)
  int KC_out;
  int* err;
};

// MODE 0: y[row][256 nt + c] = D[r][c]. MODE 1 (gate and up interleaved):
// columns [0, 128) are gate and [128, 256) up for features 128 nt + c; the
// epilogue writes silu(gate) * up as bf16 into the A image of the next GEMM.
template <int MODE>
__global__ void __launch_bounds__(PF_THREADS, 1) prefill_gemm_kernel(GemmArgs g) {
  // Persistent: one CTA per SM walks the (row tile, output tile) items with
  // the output tile varying fastest (consecutive items share their row tile's
  // A chunks in L2). Two 256-column TMEM accumulators let the epilogue of one
  // item run under the main loop of the next; the stage ring runs on across
  // items.
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* sa = base;
  uint8_t* sb = base + PF_STAGES * PF_A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + PF_STAGES * PF_B_BYTES);
  uint64_t* empty = full + PF_STAGES;
  uint64_t* acc_full = empty + PF_STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;      // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < PF_STAGES; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, 4);  // one arrival per epilogue warp
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * PF_BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int KC = g.KC, NT = g.NT;
  const int n_items = g.tiles[0] * NT;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t s = 0, ph = 0;
      for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
        const int t = w / NT, nt = w - t * NT;
        const int slot = g.tiles[3 + 3 * t];
        const uint8_t* a_src = g.A + (size_t)t * KC * PF_A_BYTES;
        const uint8_t* b_src = g.W + ((size_t)slot * NT + nt) * KC * PF_B_BYTES;
        bool ok = true;
        for (int kc = 0; kc < KC; ++kc) {
          if (!mbar_wait(empty + s, ph ^ 1, g.err, 51)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + s, PF_A_BYTES + PF_B_BYTES);
          bulk_g2s(sa + s * PF_A_BYTES, a_src + (size_t)kc * PF_A_BYTES, PF_A_BYTES, full + s);
          bulk_g2s(sb + s * PF_B_BYTES, b_src + (size_t)kc * PF_B_BYTES, PF_B_BYTES, full + s);
          if (++s == PF_STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(PF_BM, PF_BN);
      uint32_t s = 0, ph = 0, ab = 0, aph = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x) {
        if (!mbar_wait(acc_empty + ab, aph ^ 1, g.err, 54)) break;
        tc_fence_after();
        const uint32_t d = tmem + ab * PF_BN;
        for (int kc = 0; kc < KC; ++kc) {
          if (!mbar_wait(full + s, ph, g.err, 52)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(sa + s * PF_A_BYTES), b0 = smem_u32(sb + s * PF_B_BYTES);
#pragma unroll
          for (int kk = 0; kk < PF_BK / 16; ++kk)
            mma_bf16(d, smem_desc(a0 + kk * 256, 128, 1024), smem_desc(b0 + kk * 256, 128, 1024), idesc,
                     (kc | kk) != 0 ? 1u : 0u);
          tc_commit(empty + s);
          if (++s == PF_STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(acc_full + ab);
        if (++ab == 2) {
          ab = 0;
          aph ^= 1;
        }
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;
    const uint32_t lane_off = (uint32_t)(q * 32) << 16;
    uint32_t ab = 0, aph = 0;
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
      const int t = w / NT, nt = w - t * NT;
      const int row0 = g.tiles[1 + 3 * t], row1 = g.tiles[2 + 3 * t];
      if (!__all_sync(0xffffffffu, mbar_wait(acc_full + ab, aph, g.err, 53))) break;
      tc_fence_after();
      const uint32_t d = tmem + lane_off + ab * PF_BN;
      if (MODE == 1) {
        const bool live = row0 + r < row1;
        for (int j = 0; j < PF_BN / 64; ++j) {
          float gv[32], uv[32];
          tmem_ld32(d + j * 32, gv);
          tmem_ld32(d + PF_BN / 2 + j * 32, uv);
          tmem_wait_ld();
          if (j == PF_BN / 64 - 1) {  // every column of this accumulator is in registers
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + ab);
          }
          const int f0 = nt * (PF_BN / 2) + j * 32;
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float a = gv[c];
            gv[c] = (live && f0 + c < g.out) ? __fdiv_rn(a, 1.0f + expf(-a)) * uv[c] : 0.f;
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int k = f0 + u * 8;
            if (k < g.KC_out * PF_BK)
              g.a_out[((int64_t)t * g.KC_out + k / PF_BK) * (PF_A_BYTES / 16) + canon_unit(r, (k % PF_BK) / 8)] =
                  make_uint4(pack_bf16x2(gv[u * 8], gv[u * 8 + 1]), pack_bf16x2(gv[u * 8 + 2], gv[u * 8 + 3]),
                             pack_bf16x2(gv[u * 8 + 4], gv[u * 8 + 5]), pack_bf16x2(gv[u * 8 + 6], gv[u * 8 + 7]));
          }
        }
      } else {
        const int row = row0 + r;
        const int64_t y0 = (int64_t)row * g.y_ld + (int64_t)nt * PF_BN;
        float* yr = static_cast<float*>(g.y) + y0;
        uint16_t* yh = static_cast<uint16_t*>(g.y) + y0;
        const bool bf = g.y_dtype == SKCQ_DTYPE_BF16;
        const int ncol = min(PF_BN, g.out - nt * PF_BN);
        for (int j = 0; j < PF_BN / 32; ++j) {
          float v[32];
          tmem_ld32(d + j * 32, v);
          tmem_wait_ld();
          if (j == PF_BN / 32 - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty + ab);
          }
          if (row < row1) {
            if (bf) {
              if (j * 32 + 32 <= ncol && (g.y_ld & 7) == 0) {
#pragma unroll
                for (int c = 0; c < 32; c += 8)
                  *reinterpret_cast<uint4*>(yh + j * 32 + c) =
                      make_uint4(pack_bf16x2(v[c], v[c + 1]), pack_bf16x2(v[c + 2], v[c + 3]),
                                 pack_bf16x2(v[c + 4], v[c + 5]), pack_bf16x2(v[c + 6], v[c + 7]));
              } else {
                for (int c = 0; c < 32; ++c)
                  if (j * 32 + c < ncol) {
                    const __nv_bfloat16 hv = __float2bfloat16_rn(v[c]);
                    yh[j * 32 + c] = *reinterpret_cast<const uint16_t*>(&hv);
                  }
              }
            } else if (j * 32 + 32 <= ncol && (g.y_ld & 3) == 0) {
#pragma unroll
              for (int c = 0; c < 32; c += 4)
                *reinterpret_cast<float4*>(yr + j * 32 + c) = make_float4(v[c], v[c + 1], v[c + 2], v[c + 3]);
            } else {
              for (int c = 0; c < 32; ++c)
                if (j * 32 + c < ncol) yr[j * 32 + c] = v[c];
            }
          }
        }
      }
      if (++ab == 2) {
        ab = 0;
        aph ^= 1;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * PF_BN);
  }
}

static int num_sms_cached() {
  static thread_local int dev_cached = -1, sms = 148;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != dev_cached) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    dev_cached = dev;
  }
  return sms;
}

}  // namespace skcq

using namespace skcq;

extern "C" int skcq_prefill_plan(const int32_t* seg, int n_experts, int max_tiles, int32_t* tiles, void* stream) {
  SKCQ_REQUIRE(seg && tiles, SKCQ_ERR_INVALID, "prefill_plan: null pointer");
  SKCQ_REQUIRE(n_experts > 0 && max_tiles > 0, SKCQ_ERR_INVALID, "prefill_plan: %d experts, %d tiles", n_experts,
               max_tiles);
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "prefill_plan: no device error word");
  prefill_plan_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(seg, n_experts, max_tiles, tiles, err);
  return check_launch("prefill_plan");
}

extern "C" int skcq_prefill_pack(int mode, const void* x, int x_dtype, int64_t x_ld, const int32_t* row_token, int T,
                                 const float* up, int64_t up_ld, int in_dim, const int32_t* tiles, int max_tiles,
                                 void* A, void* stream) {
  SKCQ_REQUIRE(x && tiles && A, SKCQ_ERR_INVALID, "prefill_pack: null pointer");
  SKCQ_REQUIRE(mode == 0 || (mode == 1 && up), SKCQ_ERR_INVALID, "prefill_pack: mode %d", mode);
  SKCQ_REQUIRE(mode == 1 || x_dtype == SKCQ_DTYPE_F32 || x_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "prefill_pack: x dtype %d", x_dtype);
  SKCQ_REQUIRE(row_token == nullptr || T > 0, SKCQ_ERR_INVALID, "prefill_pack: token map without tokens");
  SKCQ_REQUIRE(in_dim > 0 && max_tiles > 0 && ((uintptr_t)A & 15) == 0, SKCQ_ERR_INVALID, "prefill_pack: bad sizes");
  const int KC = ceil_div(in_dim, PF_BK);
  const int64_t units = (int64_t)max_tiles * KC * 1024;
  int64_t grid = (units + 255) / 256;
  if (grid > 148 * 64) grid = 148 * 64;
  prefill_pack_kernel<<<(int)grid, 256, 0, (cudaStream_t)stream>>>(mode, x, mode == 1 ? SKCQ_DTYPE_F32 : x_dtype,
                                                                    x_ld, row_token, T, up, up_ld, in_dim, KC, tiles,
                                                                    max_tiles, static_cast<uint4*>(A));
  return check_launch("prefill_pack");
}

extern "C" int skcq_prefill_dequant(const skcq_fwd_layer* layers, int n_layers, const int32_t* active, int max_slots,
                                    int out_dim, int in_dim, int half, void* W, void* stream) {
  SKCQ_REQUIRE(layers && W, SKCQ_ERR_INVALID, "prefill_dequant: null pointer");
  SKCQ_REQUIRE(n_layers >= 1 && n_layers <= SKCQ_MAX_CODECS, SKCQ_ERR_INVALID, "prefill_dequant: %d layers",
               n_layers);
  SKCQ_REQUIRE(((uintptr_t)W & 15) == 0 && out_dim > 0 && in_dim > 0 && max_slots >= 0, SKCQ_ERR_INVALID,
               "prefill_dequant: bad sizes");
  SKCQ_REQUIRE(half >= -1 && half <= 1, SKCQ_ERR_INVALID, "prefill_dequant: half %d", half);
  DqSet set;
  set.n = n_layers;
  for (int i = 0; i < n_layers; ++i) {
    const skcq_fwd_layer& L = layers[i];
    SKCQ_REQUIRE(L.table && L.idx16 && L.bs > 0 && L.bs <= 32 && L.K > 0 && L.n_blocks >= 0, SKCQ_ERR_INVALID,
                 "prefill_dequant: layer %d incomplete or bs %d out of range", i, L.bs);
    SKCQ_REQUIRE(L.table_dtype == SKCQ_DTYPE_F32 || L.table_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
                 "prefill_dequant: layer %d table dtype %d", i, L.table_dtype);
    SKCQ_REQUIRE(L.n_blocks * L.bs + L.rem <= in_dim && (L.rem == 0 || L.remainder), SKCQ_ERR_INVALID,
                 "prefill_dequant: layer %d coverage", i);
    set.l[i] = L;
  }
  if (max_slots == 0) return SKCQ_OK;
  const int KC = ceil_div(in_dim, PF_BK), NT = ceil_div(out_dim, half < 0 ? PF_BN : PF_BN / 2);
  SKCQ_REQUIRE((int64_t)max_slots * NT < (1LL << 31) && KC < 65536, SKCQ_ERR_INVALID, "prefill_dequant: grid");
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  const int threads = half < 0 ? DQ_THREADS : DQ_THREADS / 2;
  const int smem = threads * DQ_LD * (int)sizeof(float);
  if (configured_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(prefill_dequant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         DQ_THREADS * DQ_LD * (int)sizeof(float));
    if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "prefill_dequant: %s", cudaGetErrorString(e));
    configured_dev = dev;
  }
  dim3 grid((unsigned)(max_slots * NT), (unsigned)KC);
  if (DqFastFn fast = dq_fast_pick(set)) {
    fast<<<grid, 2 * threads, 0, (cudaStream_t)stream>>>(set, active, out_dim, in_dim, NT, KC, half,
                                                         static_cast<uint4*>(W));
    return check_launch("prefill_dequant");
  }
  prefill_dequant_kernel<<<grid, threads, smem, (cudaStream_t)stream>>>(set, active, out_dim, in_dim, NT, KC, half,
                                                                      static_cast<uint4*>(W));
  return check_launch("prefill_dequant");
}

static int gemm_configure() {
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev == dev) return SKCQ_OK;
  cudaError_t e = cudaFuncSetAttribute(prefill_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(prefill_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)PF_SMEM);
  if (e != cudaSuccess) return set_error(SKCQ_ERR_CUDA, "prefill_gemm: %s", cudaGetErrorString(e));
  configured_dev = dev;
  return SKCQ_OK;
}

extern "C" int skcq_prefill_gemm(const void* A, const void* W, const int32_t* tiles, int max_tiles, int in_dim,
                                 int out_dim, void* y, int y_dtype, int64_t y_ld, void* stream) {
  SKCQ_REQUIRE(A && W && tiles && y, SKCQ_ERR_INVALID, "prefill_gemm: null pointer");
  SKCQ_REQUIRE(y_dtype == SKCQ_DTYPE_F32 || y_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "prefill_gemm: output dtype %d", y_dtype);
  SKCQ_REQUIRE(((uintptr_t)A & 15) == 0 && ((uintptr_t)W & 15) == 0, SKCQ_ERR_INVALID,
               "prefill_gemm: operands must be 16-byte aligned");
  SKCQ_REQUIRE(max_tiles > 0 && max_tiles <= 65535 && in_dim > 0 && out_dim > 0, SKCQ_ERR_INVALID,
               "prefill_gemm: bad sizes (%d row tiles)", max_tiles);
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "prefill_gemm: no device error word");
  const int rc = gemm_configure();
  if (rc != SKCQ_OK) return rc;
  GemmArgs g{static_cast<const uint8_t*>(A), static_cast<const uint8_t*>(W), tiles, ceil_div(in_dim, PF_BK),
             ceil_div(out_dim, PF_BN), out_dim, y, y_dtype, y_ld, nullptr, 0, err};
  const int64_t items = (int64_t)max_tiles * g.NT;
  const int grid = (int)std::min<int64_t>(items, num_sms_cached());
  prefill_gemm_kernel<0><<<grid, PF_THREADS, PF_SMEM, (cudaStream_t)stream>>>(g);
  return check_launch("prefill_gemm");
}

extern "C" int skcq_prefill_gemm_swiglu(const void* A, const void* W_gate_up, const int32_t* tiles, int max_tiles,
                                        int in_dim, int inter_dim, void* A_out, void* stream) {
  SKCQ_REQUIRE(A && W_gate_up && tiles && A_out, SKCQ_ERR_INVALID, "prefill_gemm_swiglu: null pointer");
  SKCQ_REQUIRE(((uintptr_t)A & 15) == 0 && ((uintptr_t)W_gate_up & 15) == 0 && ((uintptr_t)A_out & 15) == 0,
               SKCQ_ERR_INVALID, "prefill_gemm_swiglu: operands must be 16-byte aligned");
  SKCQ_REQUIRE(max_tiles > 0 && max_tiles <= 65535 && in_dim > 0 && inter_dim > 0, SKCQ_ERR_INVALID,
               "prefill_gemm_swiglu: bad sizes (%d row tiles)", max_tiles);
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "prefill_gemm_swiglu: no device error word");
  const int rc = gemm_configure();
  if (rc != SKCQ_OK) return rc;
  GemmArgs g{static_cast<const uint8_t*>(A), static_cast<const uint8_t*>(W_gate_up), tiles, ceil_div(in_dim, PF_BK),
             ceil_div(inter_dim, PF_BN / 2), inter_dim, nullptr, SKCQ_DTYPE_F32, 0, static_cast<uint4*>(A_out),
             ceil_div(inter_dim, PF_BK), err};
  const int64_t items = (int64_t)max_tiles * g.NT;
  const int grid = (int)std::min<int64_t>(items, num_sms_cached());
  prefill_gemm_kernel<1><<<grid, PF_THREADS, PF_SMEM, (cudaStream_t)stream>>>(g);
  return check_launch("prefill_gemm_swiglu");
}
