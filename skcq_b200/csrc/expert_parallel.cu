// Expert-parallel exchange for CodebookExperts.forward (skcq/codebook_experts.py:454-481)
// with experts placed across GPUs: dispatch and return over peer memory.
//
// One process per GPU. Each rank allocates one exchange buffer
// (skcq_ep_alloc) and maps every other rank's buffer through CUDA IPC
// (skcq_ep_open): plain peer loads and stores over NVLink, no multicast
// object. Rank r owns experts [bounds[r], bounds[r + 1]). A rank's buffer
// holds, per source rank s (layout in skcq_ep_layout):
//   rows[s][C][H]   the token rows s sent here (x dtype)
//   ids[s][C][kc]   per row and top-k slot: the local id of the expert when
//                   this rank owns it, else -1
//   wts[s][C][kc]   the slots' routing weights (f32)
//   cnt[s]          how many rows s sent here
//   ret[s][C][H]    what rank s returned for the rows this rank sent it: per
//                   row, the weighted sum of the outputs of s's experts
// A forward:
//   1. dispatch: every token row is written once to each rank that owns at
//      least one of its experts, at the token's position among this rank's
//      tokens bound there (ascending token order), with its slot ids/weights;
//   2. (cross-rank barrier, stream-ordered, issued by the host)
//   3. each rank computes its experts on the received rows, then writes each
//      row's weighted sum over its local slots, in ascending (expert, slot)
//      order, straight into the source rank's ret (the return is fused into the
//      combine: no separate all-to-all);
//   4. (barrier)
//   5. gather: each source adds its tokens' returned sums in ascending rank
//      order, i.e. ascending expert ranges.
// A row crosses NVLink once per destination rank, not once per slot. Every
// peer store is bounded by the capacity C the buffers were laid out for.
#include <cuda_bf16.h>

#include <cstring>

#include "common.cuh"
#include "fwd_common.cuh"

namespace skcq {

constexpr int EP_CHUNK = 1024;  // tokens per CTA when counting and placing
constexpr int EP_THREADS = 256;

struct EpLayout {
  int64_t rows, ids, wts, cnt, ret, total;
};

struct EpPeers {
  char* base[SKCQ_EP_MAX_RANKS];
  int bounds[SKCQ_EP_MAX_RANKS + 1];
};

static EpLayout ep_layout(int world, int C, int kc, int H) {
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  EpLayout L{};
  int64_t o = 0;
  const int64_t rows = (int64_t)world * C;
  L.rows = o;
  o = up(o + rows * H * 4);
  L.ids = o;
  o = up(o + rows * kc * 4);
  L.wts = o;
  o = up(o + rows * kc * 4);
  L.cnt = o;
  o = up(o + SKCQ_EP_MAX_RANKS * 4);
  L.ret = o;
  o = up(o + rows * H * 4);
  L.total = o;
  return L;
}

__device__ __forceinline__ int ep_owner(const EpPeers& p, int world, int64_t e) {
  int r = 0;
  for (int i = 1; i < world; ++i) r += (e >= p.bounds[i]) ? 1 : 0;
  return r;
}

// bit d set when rank d owns one of token t's experts; an id outside [0, E)
// is flagged (the reference's one_hot raises) and not routed
__device__ __forceinline__ unsigned ep_token_mask(const int64_t* __restrict__ topk, int t, int k, int E,
                                                  const EpPeers& p, int world, int* err) {
  unsigned m = 0;
  for (int j = 0; j < k; ++j) {
    const int64_t e = topk[(int64_t)t * k + j];
    if (e < 0 || e >= E) {
      atomicCAS(err, 0, 41);
      continue;
    }
    m |= 1u << ep_owner(p, world, e);
  }
  return m;
}

// chunk_cnt[c][d]: tokens of chunk c bound for rank d
__global__ void __launch_bounds__(EP_CHUNK) ep_count_kernel(const int64_t* __restrict__ topk, int T, int k, int E,
                                                            EpPeers p, int world, int32_t* __restrict__ chunk_cnt,
                                                            int* err) {
  __shared__ int s_cnt[SKCQ_EP_MAX_RANKS];
  if (threadIdx.x < SKCQ_EP_MAX_RANKS) s_cnt[threadIdx.x] = 0;
  __syncthreads();
  const int t = blockIdx.x * EP_CHUNK + threadIdx.x;
  const unsigned m = t < T ? ep_token_mask(topk, t, k, E, p, world, err) : 0u;
  for (int d = 0; d < world; ++d) {
    const unsigned b = __ballot_sync(0xffffffffu, (m >> d) & 1u);
    if ((threadIdx.x & 31) == 0 && b) atomicAdd(&s_cnt[d], __popc(b));
  }
  __syncthreads();
  if (threadIdx.x < SKCQ_EP_MAX_RANKS) chunk_cnt[blockIdx.x * SKCQ_EP_MAX_RANKS + threadIdx.x] = s_cnt[threadIdx.x];
}

// pos[t][d] = position of token t among this rank's tokens bound for rank d
// (-1 when none of its experts lives there); the last chunk publishes the
// totals into every destination's cnt[rank].
__global__ void __launch_bounds__(EP_CHUNK) ep_place_kernel(const int64_t* __restrict__ topk, int T, int k, int E,
                                                            EpPeers p, int world, int rank, int C, int64_t off_cnt,
                                                            const int32_t* __restrict__ chunk_cnt, int n_chunks,
                                                            int32_t* __restrict__ pos, int* err) {
  __shared__ int s_warp[EP_CHUNK / 32][SKCQ_EP_MAX_RANKS];
  __shared__ int s_base[SKCQ_EP_MAX_RANKS];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid < world) {
    int b = 0;
    for (int c = 0; c < (int)blockIdx.x; ++c) b += chunk_cnt[c * SKCQ_EP_MAX_RANKS + tid];
    s_base[tid] = b;
  }
  const int t = blockIdx.x * EP_CHUNK + tid;
  const unsigned m = t < T ? ep_token_mask(topk, t, k, E, p, world, err) : 0u;
  unsigned ballots[SKCQ_EP_MAX_RANKS];
#pragma unroll
  for (int d = 0; d < SKCQ_EP_MAX_RANKS; ++d) {
    ballots[d] = 0u;
    if (d < world) {
      ballots[d] = __ballot_sync(0xffffffffu, (m >> d) & 1u);
      if (lane == 0) s_warp[w][d] = __popc(ballots[d]);
    }
  }
  __syncthreads();
  if (tid < world) {
    int run = 0;
    for (int i = 0; i < EP_CHUNK / 32; ++i) {
      const int c = s_warp[i][tid];
      s_warp[i][tid] = run;
      run += c;
    }
    if ((int)blockIdx.x == n_chunks - 1) {
      int total = s_base[tid] + run;
      if (total > C) {
        atomicCAS(err, 0, 62);
        total = C;
      }
      reinterpret_cast<int32_t*>(p.base[tid] + off_cnt)[rank] = total;
    }
  }
  __syncthreads();
  if (t < T) {
#pragma unroll
    for (int d = 0; d < SKCQ_EP_MAX_RANKS; ++d) {
      if (d < world) {
        int v = -1;
        if ((m >> d) & 1u) v = s_base[d] + s_warp[w][d] + __popc(ballots[d] & ((1u << lane) - 1u));
        pos[(int64_t)t * world + d] = v;
      }
    }
  }
}

// One CTA per token (grid-stride): the row is read once and stored to every
// destination rank, then the slots' ids and weights.
__global__ void __launch_bounds__(EP_THREADS) ep_send_kernel(const void* __restrict__ x, int esz, int64_t x_ld,
                                                             int vec16, const int64_t* __restrict__ topk,
                                                             const void* __restrict__ w, int w_dtype, int T, int k,
                                                             int E, EpPeers p, int world, int rank, int C, int H,
                                                             int kc, EpLayout lay, const int32_t* __restrict__ pos,
                                                             int* err) {
  __shared__ int s_pos[SKCQ_EP_MAX_RANKS];
  const int64_t row_bytes = (int64_t)H * esz;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    if (threadIdx.x < world) {
      int v = pos[(int64_t)t * world + threadIdx.x];
      if (v >= C) {
        atomicCAS(err, 0, 62);
        v = -1;
      }
      s_pos[threadIdx.x] = v;
    }
    __syncthreads();
    const char* src = static_cast<const char*>(x) + (int64_t)t * x_ld * esz;
    if (vec16) {
      const int nv = (int)(row_bytes / 16);
      for (int v = threadIdx.x; v < nv; v += blockDim.x) {
        const uint4 val = reinterpret_cast<const uint4*>(src)[v];
        for (int d = 0; d < world; ++d) {
          const int q = s_pos[d];
          if (q < 0) continue;
          reinterpret_cast<uint4*>(p.base[d] + lay.rows + ((int64_t)rank * C + q) * row_bytes)[v] = val;
        }
      }
    } else if (esz == 2) {
      for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const uint16_t val = reinterpret_cast<const uint16_t*>(src)[i];
        for (int d = 0; d < world; ++d) {
          const int q = s_pos[d];
          if (q < 0) continue;
          reinterpret_cast<uint16_t*>(p.base[d] + lay.rows + ((int64_t)rank * C + q) * row_bytes)[i] = val;
        }
      }
    } else {
      for (int i = threadIdx.x; i < H; i += blockDim.x) {
        const uint32_t val = reinterpret_cast<const uint32_t*>(src)[i];
        for (int d = 0; d < world; ++d) {
          const int q = s_pos[d];
          if (q < 0) continue;
          reinterpret_cast<uint32_t*>(p.base[d] + lay.rows + ((int64_t)rank * C + q) * row_bytes)[i] = val;
        }
      }
    }
    if (threadIdx.x < k) {
      const int j = threadIdx.x;
      const int64_t e = topk[(int64_t)t * k + j];
      const float wt = ld_any(w, (int64_t)t * k + j, w_dtype);
      const int own = (e >= 0 && e < E) ? ep_owner(p, world, e) : -1;
      for (int d = 0; d < world; ++d) {
        const int q = s_pos[d];
        if (q < 0) continue;
        const int64_t slot = ((int64_t)rank * C + q) * kc + j;
        reinterpret_cast<int32_t*>(p.base[d] + lay.ids)[slot] = own == d ? (int)(e - p.bounds[d]) : -1;
        reinterpret_cast<float*>(p.base[d] + lay.wts)[slot] = wt;
      }
    }
    __syncthreads();
  }
}

// Received rows as a (world * C, k) routing of the local experts: rows past a
// source's count and slots owned elsewhere get id -1 (weight 0).
__global__ void ep_unpack_kernel(const char* __restrict__ buf, EpLayout lay, int world, int C, int k, int kc,
                                 int64_t* __restrict__ topk_out, float* __restrict__ w_out) {
  const int32_t* cnt = reinterpret_cast<const int32_t*>(buf + lay.cnt);
  const int32_t* ids = reinterpret_cast<const int32_t*>(buf + lay.ids);
  const float* wts = reinterpret_cast<const float*>(buf + lay.wts);
  const int64_t total = (int64_t)world * C * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % k);
    const int64_t row = i / k;
    const int s = (int)(row / C);
    const int r = (int)(row - (int64_t)s * C);
    int n = cnt[s];
    n = n < 0 ? 0 : (n > C ? C : n);
    const bool live = r < n;
    const int64_t src = row * kc + j;
    topk_out[i] = live ? (int64_t)ids[src] : -1;
    w_out[i] = live ? wts[src] : 0.f;
  }
}

// For every received row (r = s * C + i, i < cnt[s]): the weighted sum over
// its local slots, in ascending (expert, slot) order, of the pair outputs
// (sum over splits of part[split][row_of_pair[kpos * world * C + r]]), stored
// into rank s's ret[rank][i]. The slot order is resolved once per CTA in
// shared memory, as skcq_combine does.
__global__ void __launch_bounds__(EP_THREADS) ep_return_kernel(const void* __restrict__ part, int part_dtype,
                                                               int n_split, int64_t P,
                                                               const int32_t* __restrict__ row_of_pair,
                                                               const int64_t* __restrict__ topk,
                                                               const float* __restrict__ w, const char* buf,
                                                               EpPeers p, EpLayout lay, int world, int rank, int C,
                                                               int k, int H, int out_dtype, int vec8) {
  __shared__ int s_row[32];
  __shared__ float s_w[32];
  __shared__ int s_n;
  const int32_t* cnt = reinterpret_cast<const int32_t*>(buf + lay.cnt);
  const int Tl = world * C;
  const int64_t stride = P * H;
  for (int r = blockIdx.x; r < Tl; r += gridDim.x) {
    const int s = r / C, i = r - s * C;
    int n = cnt[s];
    n = n < 0 ? 0 : (n > C ? C : n);
    if (i >= n) continue;  // the same for every thread of the CTA
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      int64_t e = lane < k ? topk[(int64_t)r * k + lane] : INT64_MAX;
      if (e < 0) e = INT64_MAX;
      int rk = 0;
      for (int j = 0; j < k; ++j) {
        const int64_t ej = __shfl_sync(0xffffffffu, e, j);
        rk += (ej < e || (ej == e && j < lane)) ? 1 : 0;
      }
      const unsigned live = __ballot_sync(0xffffffffu, lane < k && e != INT64_MAX);
      if (lane == 0) s_n = __popc(live);
      if (lane < k) {
        s_row[rk] = row_of_pair[(int64_t)lane * Tl + r];
        s_w[rk] = w[(int64_t)r * k + lane];
      }
    }
    __syncthreads();
    const int n_live = s_n;
    char* dst = p.base[s] + lay.ret;
    const int64_t o0 = ((int64_t)rank * C + i) * H;
    if (vec8) {  // bf16 pair outputs, one split, H % 8 == 0: 16-byte accesses
      for (int h = (blockIdx.y * EP_THREADS + threadIdx.x) * 8; h < H; h += gridDim.y * EP_THREADS * 8) {
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
        st_x8(dst, o0 + h, out_dtype, acc);
      }
    } else {
      for (int h = blockIdx.y * EP_THREADS + threadIdx.x; h < H; h += gridDim.y * EP_THREADS) {
        float acc = 0.f;
        for (int step = 0; step < n_live; ++step) {
          const int64_t q = (int64_t)s_row[step] * H + h;
          float y = ld_any(part, q, part_dtype);
          for (int sp = 1; sp < n_split; ++sp) y += ld_any(part, sp * stride + q, part_dtype);
          acc = __fadd_rn(acc, __fmul_rn(y, s_w[step]));
        }
        st_any(dst, o0 + h, out_dtype, acc);
      }
    }
    __syncthreads();
  }
}

// out[t][h] = sum over ranks d ascending with pos[t][d] >= 0 of ret[d][pos][h]
__global__ void __launch_bounds__(EP_THREADS) ep_gather_kernel(const char* __restrict__ buf, EpLayout lay,
                                                               const int32_t* __restrict__ pos, int T, int world,
                                                               int C, int H, int ret_dtype, void* __restrict__ out,
                                                               int out_dtype, int vec8) {
  __shared__ int s_pos[SKCQ_EP_MAX_RANKS];
  const void* ret = buf + lay.ret;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    if (threadIdx.x < world) {
      const int v = pos[(int64_t)t * world + threadIdx.x];
      s_pos[threadIdx.x] = (v >= 0 && v < C) ? v : -1;
    }
    __syncthreads();
    if (vec8) {  // bf16 returned sums, H % 8 == 0: 16-byte accesses
      for (int h = (blockIdx.y * EP_THREADS + threadIdx.x) * 8; h < H; h += gridDim.y * EP_THREADS * 8) {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int d = 0; d < world; ++d) {
          const int q = s_pos[d];
          if (q < 0) continue;
          float y[8];
          ld_bf16x8(ret, ((int64_t)d * C + q) * H + h, y);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += y[j];
        }
        st_x8(out, (int64_t)t * H + h, out_dtype, acc);
      }
    } else {
      for (int h = blockIdx.y * EP_THREADS + threadIdx.x; h < H; h += gridDim.y * EP_THREADS) {
        float acc = 0.f;
        for (int d = 0; d < world; ++d) {
          const int q = s_pos[d];
          if (q >= 0) acc += ld_any(ret, ((int64_t)d * C + q) * H + h, ret_dtype);
        }
        st_any(out, (int64_t)t * H + h, out_dtype, acc);
      }
    }
    __syncthreads();
  }
}

static bool ep_sizes_ok(int world, int rank, int C, int kc, int H) {
  return world >= 1 && world <= SKCQ_EP_MAX_RANKS && rank >= 0 && rank < world && C >= 1 && kc >= 1 && kc <= 31 &&
         H >= 1 && (int64_t)world * C * kc < (1LL << 31) && (int64_t)world * C < (1LL << 31);
}

static dim3 ep_row_grid(int rows, int H, int vec8) {
  const int gx = rows < 148 * 16 ? (rows < 1 ? 1 : rows) : 148 * 16;
  int gy = ceil_div(vec8 ? H / 8 : H, EP_THREADS);
  const int want_y = ceil_div(148 * 4, gx);
  if (gy > want_y) gy = want_y;
  return dim3(gx, gy < 1 ? 1 : gy);
}

}  // namespace skcq

using namespace skcq;

extern "C" int skcq_ep_layout(int world, int capacity, int top_k_cap, int hidden, int64_t* offsets) {
  SKCQ_REQUIRE(offsets, SKCQ_ERR_INVALID, "ep_layout: null pointer");
  SKCQ_REQUIRE(ep_sizes_ok(world, 0, capacity, top_k_cap, hidden), SKCQ_ERR_INVALID,
               "ep_layout: bad sizes (world %d, capacity %d, top-k %d, hidden %d)", world, capacity, top_k_cap,
               hidden);
  const EpLayout L = ep_layout(world, capacity, top_k_cap, hidden);
  offsets[0] = L.rows;
  offsets[1] = L.ids;
  offsets[2] = L.wts;
  offsets[3] = L.cnt;
  offsets[4] = L.ret;
  offsets[5] = L.total;
  return SKCQ_OK;
}

extern "C" int skcq_ep_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  SKCQ_REQUIRE(ptr && ipc_handle && bytes > 0, SKCQ_ERR_INVALID, "ep_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  SKCQ_REQUIRE(e == cudaSuccess, SKCQ_ERR_CUDA, "ep_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) {
    cudaIpcMemHandle_t h;
    e = cudaIpcGetMemHandle(&h, p);
    if (e == cudaSuccess) memcpy(ipc_handle, &h, sizeof(h));
  }
  if (e != cudaSuccess) {
    cudaFree(p);
    SKCQ_REQUIRE(false, SKCQ_ERR_CUDA, "ep_alloc: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return SKCQ_OK;
}

extern "C" int skcq_ep_open(const void* ipc_handle, void** ptr) {
  SKCQ_REQUIRE(ipc_handle && ptr, SKCQ_ERR_INVALID, "ep_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  SKCQ_REQUIRE(e == cudaSuccess, SKCQ_ERR_CUDA, "ep_open: %s", cudaGetErrorString(e));
  *ptr = p;
  return SKCQ_OK;
}

extern "C" int skcq_ep_close(void* ptr) {
  SKCQ_REQUIRE(ptr, SKCQ_ERR_INVALID, "ep_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  SKCQ_REQUIRE(e == cudaSuccess, SKCQ_ERR_CUDA, "ep_close: %s", cudaGetErrorString(e));
  return SKCQ_OK;
}

extern "C" int skcq_ep_free(void* ptr) {
  SKCQ_REQUIRE(ptr, SKCQ_ERR_INVALID, "ep_free: null pointer");
  const cudaError_t e = cudaFree(ptr);
  SKCQ_REQUIRE(e == cudaSuccess, SKCQ_ERR_CUDA, "ep_free: %s", cudaGetErrorString(e));
  return SKCQ_OK;
}

static int ep_peers(const int32_t* bounds, void* const* peers, int world, int n_experts, EpPeers* out) {
  SKCQ_REQUIRE(bounds && peers, SKCQ_ERR_INVALID, "ep: null bounds or peers");
  SKCQ_REQUIRE(bounds[0] == 0 && bounds[world] == n_experts, SKCQ_ERR_INVALID,
               "ep: expert bounds [%d, %d] do not cover %d experts", bounds[0], bounds[world], n_experts);
  for (int r = 0; r < SKCQ_EP_MAX_RANKS; ++r) out->base[r] = nullptr;
  for (int r = 0; r <= SKCQ_EP_MAX_RANKS; ++r) out->bounds[r] = n_experts;
  for (int r = 0; r < world; ++r) {
    SKCQ_REQUIRE(peers[r] && ((uintptr_t)peers[r] & 255) == 0, SKCQ_ERR_INVALID, "ep: buffer of rank %d", r);
    SKCQ_REQUIRE(bounds[r + 1] >= bounds[r], SKCQ_ERR_INVALID, "ep: expert bounds not ascending at rank %d", r);
    out->base[r] = static_cast<char*>(peers[r]);
  }
  for (int r = 0; r <= world; ++r) out->bounds[r] = bounds[r];
  return SKCQ_OK;
}

extern "C" int skcq_ep_dispatch(const void* x, int x_dtype, int64_t x_ld, const int64_t* topk, const void* weights,
                                int w_dtype, int T, int k, int n_experts, const int32_t* bounds, void* const* peers,
                                int world, int rank, int capacity, int top_k_cap, int hidden, int32_t* chunk_counts,
                                int32_t* pos, void* stream) {
  SKCQ_REQUIRE(ep_sizes_ok(world, rank, capacity, top_k_cap, hidden), SKCQ_ERR_INVALID,
               "ep_dispatch: bad sizes (world %d, rank %d, capacity %d, top-k %d, hidden %d)", world, rank, capacity,
               top_k_cap, hidden);
  SKCQ_REQUIRE(T >= 0 && T <= capacity && k >= 1 && k <= top_k_cap && n_experts >= world, SKCQ_ERR_INVALID,
               "ep_dispatch: %d tokens (capacity %d), top-k %d (cap %d), %d experts", T, capacity, k, top_k_cap,
               n_experts);
  SKCQ_REQUIRE(chunk_counts && (T == 0 || (x && topk && weights && pos)), SKCQ_ERR_INVALID, "ep_dispatch: null pointer");
  SKCQ_REQUIRE(x_dtype == SKCQ_DTYPE_F32 || x_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID, "ep_dispatch: x dtype %d",
               x_dtype);
  SKCQ_REQUIRE(w_dtype == SKCQ_DTYPE_F32 || w_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "ep_dispatch: weight dtype %d", w_dtype);
  SKCQ_REQUIRE(x_ld >= hidden || T == 0, SKCQ_ERR_INVALID, "ep_dispatch: row stride %lld", (long long)x_ld);
  EpPeers p;
  const int rc = ep_peers(bounds, peers, world, n_experts, &p);
  if (rc != SKCQ_OK) return rc;
  int* err = device_error_word();
  SKCQ_REQUIRE(err != nullptr, SKCQ_ERR_CUDA, "ep_dispatch: no device error word");
  const EpLayout lay = ep_layout(world, capacity, top_k_cap, hidden);
  const int esz = x_dtype == SKCQ_DTYPE_BF16 ? 2 : 4;
  const int n_chunks = T > 0 ? ceil_div(T, EP_CHUNK) : 1;
  cudaStream_t s = (cudaStream_t)stream;
  ep_count_kernel<<<n_chunks, EP_CHUNK, 0, s>>>(topk, T, k, n_experts, p, world, chunk_counts, err);
  ep_place_kernel<<<n_chunks, EP_CHUNK, 0, s>>>(topk, T, k, n_experts, p, world, rank, capacity, lay.cnt,
                                                chunk_counts, n_chunks, pos, err);
  if (T > 0) {
    const int vec16 = ((int64_t)hidden * esz) % 16 == 0 && ((uintptr_t)x & 15) == 0 && (x_ld * esz) % 16 == 0;
    const int grid = T < 148 * 8 ? T : 148 * 8;
    ep_send_kernel<<<grid, EP_THREADS, 0, s>>>(x, esz, x_ld, vec16, topk, weights, w_dtype, T, k, n_experts, p, world,
                                               rank, capacity, hidden, top_k_cap, lay, pos, err);
  }
  return check_launch("ep_dispatch");
}

extern "C" int skcq_ep_unpack(const void* buffer, int world, int capacity, int k, int top_k_cap, int hidden,
                              int64_t* topk_out, float* weights_out, void* stream) {
  SKCQ_REQUIRE(buffer && topk_out && weights_out, SKCQ_ERR_INVALID, "ep_unpack: null pointer");
  SKCQ_REQUIRE(ep_sizes_ok(world, 0, capacity, top_k_cap, hidden) && k >= 1 && k <= top_k_cap, SKCQ_ERR_INVALID,
               "ep_unpack: bad sizes");
  const EpLayout lay = ep_layout(world, capacity, top_k_cap, hidden);
  const int64_t total = (int64_t)world * capacity * k;
  int64_t grid = (total + 255) / 256;
  if (grid > 148 * 16) grid = 148 * 16;
  ep_unpack_kernel<<<(int)grid, 256, 0, (cudaStream_t)stream>>>(static_cast<const char*>(buffer), lay, world,
                                                                capacity, k, top_k_cap, topk_out, weights_out);
  return check_launch("ep_unpack");
}

extern "C" int skcq_ep_return(const void* part, int part_dtype, int n_split, int64_t P, const int32_t* row_of_pair,
                              const int64_t* topk_local, const float* weights_local, const void* buffer,
                              void* const* peers, const int32_t* bounds, int n_experts, int world, int rank,
                              int capacity, int k, int top_k_cap, int hidden, int out_dtype, void* stream) {
  SKCQ_REQUIRE(part && row_of_pair && topk_local && weights_local && buffer, SKCQ_ERR_INVALID,
               "ep_return: null pointer");
  SKCQ_REQUIRE(ep_sizes_ok(world, rank, capacity, top_k_cap, hidden) && k >= 1 && k <= top_k_cap && n_split >= 1,
               SKCQ_ERR_INVALID, "ep_return: bad sizes");
  SKCQ_REQUIRE(P == (int64_t)world * capacity * k, SKCQ_ERR_INVALID, "ep_return: %lld pairs for %d x %d rows x %d",
               (long long)P, world, capacity, k);
  SKCQ_REQUIRE(part_dtype == SKCQ_DTYPE_F32 || part_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "ep_return: pair-output dtype %d", part_dtype);
  SKCQ_REQUIRE(out_dtype == SKCQ_DTYPE_F32 || out_dtype == SKCQ_DTYPE_BF16, SKCQ_ERR_INVALID,
               "ep_return: output dtype %d", out_dtype);
  EpPeers p;
  const int rc = ep_peers(bounds, peers, world, n_experts, &p);
  if (rc != SKCQ_OK) return rc;
  const EpLayout lay = ep_layout(world, capacity, top_k_cap, hidden);
  const int vec8 = part_dtype == SKCQ_DTYPE_BF16 && n_split == 1 && hidden % 8 == 0 && ((uintptr_t)part & 15) == 0;
  ep_return_kernel<<<ep_row_grid(world * capacity, hidden, vec8), EP_THREADS, 0, (cudaStream_t)stream>>>(
      part, part_dtype, n_split, P, row_of_pair, topk_local, weights_local, static_cast<const char*>(buffer), p, lay,
      world, rank, capacity, k, hidden, out_dtype, vec8);
  return check_launch("ep_return");
}

extern "C" int skcq_ep_gather(const void* buffer, const int32_t* pos, int T, int world, int capacity, int top_k_cap,
                              int hidden, int ret_dtype, void* out, int out_dtype, void* stream) {
  SKCQ_REQUIRE(buffer && (T == 0 || (pos && out)), SKCQ_ERR_INVALID, "ep_gather: null pointer");
  SKCQ_REQUIRE(ep_sizes_ok(world, 0, capacity, top_k_cap, hidden) && T >= 0 && T <= capacity, SKCQ_ERR_INVALID,
               "ep_gather: bad sizes");
  SKCQ_REQUIRE((ret_dtype == SKCQ_DTYPE_F32 || ret_dtype == SKCQ_DTYPE_BF16) &&
                   (out_dtype == SKCQ_DTYPE_F32 || out_dtype == SKCQ_DTYPE_BF16),
               SKCQ_ERR_INVALID, "ep_gather: dtypes %d, %d", ret_dtype, out_dtype);
  if (T == 0) return SKCQ_OK;
  const EpLayout lay = ep_layout(world, capacity, top_k_cap, hidden);
  const int vec8 = ret_dtype == SKCQ_DTYPE_BF16 && hidden % 8 == 0 && ((uintptr_t)out & 15) == 0;
  ep_gather_kernel<<<ep_row_grid(T, hidden, vec8), EP_THREADS, 0, (cudaStream_t)stream>>>(
      static_cast<const char*>(buffer), lay, pos, T, world, capacity, hidden, ret_dtype, out, out_dtype, vec8);
  return check_launch("ep_gather");
}
