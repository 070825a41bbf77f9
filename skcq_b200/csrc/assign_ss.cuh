// Shared-memory-operand assignment kernel (assign_ss.cu), launched by
// skcq_assign for packed widths of three or more MMA k-steps.
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace skcq {

// Writes -(g + 1) (the winning 32-centroid group g, not yet re-scored) into
// group[b][i] for every live point; n_pad % 256 == 0, k_pad % 128 == 0,
// kp % 8 == 0 and kp <= 64. Returns the launch status.
cudaError_t assign_ss_launch(const float* A, const float* B, int nblk, int n_pad, int k_pad, int kp,
                             const int32_t* n, const int32_t* k, const int32_t* active, int32_t* group, int* err,
                             int grid, cudaStream_t s);

}  // namespace skcq
