/*
 * skcq_b200 -- C ABI of the B200 (sm_100a) kernels behind the SKCQ codebook
 * build and codebook-expert forward paths.
 *
 * Conventions (every entry point):
 *   - plain pointers and sizes, no framework types; all data pointers are
 *     DEVICE pointers unless documented as host;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy stream); calls
 *     are stream-ordered and asynchronous;
 *   - return 0 (SKCQ_OK) or a negative status; skcq_last_error() returns the
 *     message of the calling thread's most recent failure. Nothing throws.
 *
 * The reference (levzlotnik/SKCQ) is pure Python/PyTorch; each entry point
 * below names the reference function whose device work it replaces.
 *
 * Layout vocabulary for one k-means "problem set" (nblk independent
 * problems of dimension bs, e.g. one per column block of a weight matrix):
 *   X [nblk][n_pad][bs]  f32  assignment points (cosine: unit rows)
 *   R [nblk][n_pad][bs]  f32  update points (cosine: raw rows; l2: = X)
 *   C [nblk][k_pad][bs]  f32  centroids
 *   n[nblk], k[nblk]     i32  valid points / centroids of each problem
 *   active[nblk]         i32  1 while the problem still iterates
 *   labels [nblk][n_pad] i32
 * n_pad is a multiple of SKCQ_ROWS_PER_UNIT and k_pad of SKCQ_CENT_TILE.
 * metric: 0 = cosine (maximise x.c), 1 = euclidean (minimise ||c||^2 - 2 x.c).
 */
#ifndef SKCQ_B200_H
#define SKCQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SKCQ_OK 0
#define SKCQ_ERR_INVALID (-1)     /* bad argument: size, alignment, null pointer */
#define SKCQ_ERR_CUDA (-2)        /* CUDA runtime / launch error */
#define SKCQ_ERR_DEVICE (-3)      /* a device-side check or bounded wait failed */
#define SKCQ_ERR_FLIP_INDEX (-5)  /* spherical flip label >= block size (IndexError in the reference) */

#define SKCQ_METRIC_COSINE 0
#define SKCQ_METRIC_L2 1

#define SKCQ_ROWS_PER_UNIT 256 /* rows of points one assignment work unit owns */
#define SKCQ_CENT_TILE 128     /* centroids per tensor-core tile */

/* Copies the calling thread's last error message into buf (NUL-terminated). */
int skcq_last_error(char* buf, size_t len);
/* ABI version of this library (bumped on any signature change). */
int skcq_abi_version(void);

/* Device error codes of skcq_poll_device_error whose cause is a bounded wait
 * that ran out (a pipeline partner that did not arrive within ~2 s): a
 * tensor-core assignment wait (11-17), a prefill GEMM wait (51-54) or the
 * self-test below. The kernel returned; the context stays usable. */
#define SKCQ_DEVICE_CODE_SELFTEST 90

/* Self-test of that path: launches one thread that waits on a barrier nothing
 * arrives on, for at most limit_clocks SM clocks (<= 4e9), through the same
 * bounded wait the kernels use; it records SKCQ_DEVICE_CODE_SELFTEST and
 * returns. A later skcq_poll_device_error reports SKCQ_ERR_DEVICE with that
 * code and clears it. */
int skcq_selftest_wait_timeout(long long limit_clocks, void* stream);
/* Synchronises `stream`, then returns SKCQ_ERR_DEVICE (and clears the word) if
 * any kernel recorded a device-side failure (a bounded wait that gave up, an
 * inconsistent reseed selection), else SKCQ_OK. */
int skcq_poll_device_error(void* stream);

/* Packed operand width: tf32 columns per point/centroid for the split-precision
 * tensor-core assignment (3*bs products, +2 bias columns for euclidean, rounded
 * up to the tf32 MMA K of 8). Host-side helper, no device work. */
int skcq_packed_width(int metric, int bs);

/* ---- point preparation (skcq/codebook/spherical.py:243-262,
 *      skcq/codebook/euclidean.py:455-478: block zero test and compaction) --- */

/* For each problem, lists the source points whose block norm is >= thr (all
 * points when skip_zeros == 0) in ascending order into rowmap[b][*] and their
 * count into n_out[b]. Source point p of problem b is row p, columns
 * [b*bs, b*bs+bs) of W (row-major, leading dimension ld); with shared != 0 there
 * is one problem whose point p is row p / n_blocks, block p % n_blocks. */
int skcq_compact_points(const float* W, int64_t ld, int n_rows, int bs, int n_blocks, int shared, float thr,
                        int skip_zeros, int nblk, int npts_pad, int32_t* rowmap, int32_t* n_out, void* stream);

/* Gathers the listed points: R[b][i] = point(rowmap[b][i]) and
 * X[b][i] = normalize(R[b][i]) (normalize != 0, F.normalize eps 1e-12) or = R.
 * Rows i >= n[b] are zero-filled. R may be NULL. */
int skcq_gather_points(const float* W, int64_t ld, int bs, int n_blocks, int shared, int nblk, const int32_t* rowmap,
                       const int32_t* n, int n_pad, int normalize, float* X, float* R, void* stream);

/* Writes the split-tf32 tensor-core operand of the points
 * (A[nblk][n_pad/8][kp/4][8][4], kp = skcq_packed_width). */
int skcq_pack_points(int metric, const float* X, int nblk, int n_pad, int bs, float* A, void* stream);

/* C[b][c] = X[b][perm[b][c]] for c < k[b]: the Forgy initialisation of
 * skcq/codebook/kmeans.py:201-202 given torch.randperm's draw. */
int skcq_init_from_points(const float* X, int n_pad, int bs, int nblk, const int64_t* perm, int64_t perm_ld,
                          const int32_t* k, int k_pad, float* C, void* stream);

/* ---- Lloyd iteration (skcq/codebook/kmeans.py:136-249) --------------------- */

/* Writes the split-tf32 operand of the centroids (B[nblk][k_pad/8][kp/4][8][4];
 * euclidean adds -||c||^2/2 as two bias columns) and cnorm[b][c] = ||c||^2
 * (kmeans.py:59). Problems with active[b] == 0 are skipped. */
int skcq_pack_centroids(int metric, const float* C, int nblk, int k_pad, int bs, const int32_t* k,
                        const int32_t* active, float* B, float* cnorm, void* stream);

/* Nearest centroid of every point of every active problem: assign_cosine /
 * assign_l2 (kmeans.py:25-66). tcgen05 kind::tf32 GEMM of the split operands
 * with the arg-max fused into the tensor-memory epilogue; the winning group of
 * 32 centroids is re-scored in exact fp32 with the reference formula. */
int skcq_assign(int metric, const float* A, const float* B, const float* X, const float* C, const float* cnorm,
                int nblk, int n_pad, int k_pad, int bs, const int32_t* n, const int32_t* k, const int32_t* active,
                int32_t* labels, void* stream);

/* Euclidean problems of block size 2-4 (replaces the full scan of assign_l2,
 * skcq/codebook/kmeans.py:46-66, for low-dimensional codebooks): the labels
 * skcq_assign_exact gives (the reference formula's arg-max over all k[b]
 * centroids, first maximum), found through a grid of G cells per coordinate
 * (boundaries at quantiles of the centroids). Each point is scored against
 * the centroids of its cell neighbourhood and certified when every other
 * centroid provably scores lower (distance bound plus the fp32 rounding
 * bound); a point left uncertified is searched again over the boxes of
 * radius 2 .. ring_max cells around its own cell (ring_max 0: no such
 * search; at most 3). Certified points get labels[b][i] and unres[b][i] = 0;
 * the others unres[b][i] = 1 and their labels are left as they were (search
 * them over all centroids). Requires 2 <= bs <= 4, 2 <= G <= 256,
 * bs * (G - 1) <= 1024, G^bs <= 2^20; scratch (256-byte aligned) of
 * skcq_assign_grid_scratch_bytes(nblk, n_pad, k_pad, bs, G) bytes. cnorm as
 * skcq_pack_centroids writes it. */
size_t skcq_assign_grid_scratch_bytes(int nblk, int n_pad, int k_pad, int bs, int G);
int skcq_assign_grid(const float* X, const float* C, const float* cnorm, int nblk, int n_pad, int k_pad, int bs,
                     const int32_t* n, const int32_t* k, const int32_t* active, int G, int ring_max,
                     int32_t* labels, uint8_t* unres, void* scratch, size_t scratch_bytes, void* stream);

/* Same contract as skcq_assign, computed with fp32 FMAs on CUDA cores over all
 * centroids (the reference formula everywhere). Used to cross-check. */
int skcq_assign_exact(int metric, const float* X, const float* C, const float* cnorm, int nblk, int n_pad, int k_pad,
                      int bs, const int32_t* n, const int32_t* k, const int32_t* active, int32_t* labels,
                      void* stream);

/* Segmented sums and counts of the update (kmeans.py:152-159 / 210-217):
 * sums[b][labels[b][i]] += R[b][i], counts[b][labels[b][i]] += 1.
 * sums/counts must be zero on entry (skcq_finalize leaves them zeroed).
 * changed (optional, from skcq_mark_changed): points of clusters with
 * changed == 0 are counted but not summed (skcq_finalize keeps those
 * centroids and ignores their sums). */
int skcq_update(const float* R, const int32_t* labels, int nblk, int n_pad, int k_pad, int bs, const int32_t* n,
                const int32_t* k, const int32_t* active, float* sums, int32_t* counts, const uint8_t* changed,
                void* stream);

/* Empty-cluster reseed (kmeans.py:161-172, 219-230): for each active problem
 * with empty clusters, the n_empty worst-fit points (cosine: lowest
 * <x, c_label>; euclidean: largest ||x - c_label||^2; ties by point index)
 * are written, in that order, into the sums of the empty clusters in
 * ascending cluster order. n_empty[b] receives the count. `scratch` must hold
 * skcq_reseed_scratch_bytes(nblk, k_pad) bytes. k_pad must be a multiple of
 * SKCQ_CENT_TILE and at most 1048576 (skcq_reseed_scratch_bytes returns 0
 * beyond that). */
size_t skcq_reseed_scratch_bytes(int nblk, int k_pad);
int skcq_reseed(int metric, const float* X, const float* C, const int32_t* labels, int nblk, int n_pad, int k_pad,
                int bs, const int32_t* n, const int32_t* k, const int32_t* active, float* sums,
                const int32_t* counts, int32_t* n_empty, void* scratch, void* stream);

/* Same result as skcq_reseed, for callers that cannot allocate device memory:
 * hosts that give the whole device to their own allocator and forbid
 * cudaMalloc, or plug-in interfaces that only hand over the step's inputs and
 * outputs. No counterpart in the reference (which lets torch allocate).
 * The scratch is a 16 MiB array compiled into the library, held by every GPU
 * that loads it until the process exits; problems with k_pad above 1048576
 * are rejected with SKCQ_ERR_INVALID. The first call on a device looks up the
 * array's device address (make that first call before any stream capture);
 * the address is cached for the life of the process, so the entry point must
 * not be used across a cudaDeviceReset. k_pad must be a multiple of
 * SKCQ_CENT_TILE (as for skcq_reseed).
 * All calls share the array: the kernel writes every scratch word before
 * reading it, so no state carries over, but calls that overlap on the GPU
 * (e.g. on two streams) race and must be serialised by the caller. Allocates
 * nothing (cudaMemsetAsync of n_empty only). */
int skcq_reseed_noalloc(int metric, const float* X, const float* C, const int32_t* labels, int nblk, int n_pad,
                        int k_pad, int bs, const int32_t* n, const int32_t* k, const int32_t* active, float* sums,
                        const int32_t* counts, int32_t* n_empty, void* stream);

/* Reseed for row-sharded problems (each rank holds a slice of every problem's
 * points; sums/counts already summed over ranks). For each active problem
 * with empty clusters (from the global `counts`), writes this rank's
 * min(n_empty, n[b]) worst-fit points, worst first, using the reseed order of
 * skcq_reseed with the point's global index gofs[b] + i breaking ties:
 * keys[b][e] = (score key << 32 | global index) ^ 2^63 (so signed int64 order
 * is the selection order) and vecs[b][e][:] = X[b][i]. keys must be
 * pre-filled with INT64_MAX and vecs with 0 ([nblk][m_max] / [nblk][m_max][bs],
 * m_max >= every n_empty); n_empty[b] receives the count. Merging the ranks'
 * lists and taking the n_empty smallest keys gives the single-process choice.
 * scratch as for skcq_reseed. */
int skcq_reseed_candidates(int metric, const float* X, const float* C, const int32_t* labels, int nblk, int n_pad,
                           int k_pad, int bs, const int32_t* n, const int32_t* k, const int32_t* active,
                           const int32_t* counts, const int64_t* gofs, int m_max, int64_t* keys, float* vecs,
                           int32_t* n_empty, void* scratch, void* stream);

/* New centroids, movement and convergence (kmeans.py:174-188, 231-244):
 * cosine C = normalize(sums); euclidean C = sums / counts (reseeded clusters
 * take the point). moved = ||C_new - C_old||_F; a problem whose moved < 1e-6
 * stops (active = 0, converged = 1). Records moved_hist[iter][b] and
 * nempty_hist[iter][b], sets iters_run[b] = iter + 1, and zeroes sums/counts.
 * changed (optional, [nblk][k_pad] bytes from skcq_mark_changed): a non-empty
 * cluster with changed == 0 has the same members as at the previous update,
 * so its centroid is kept bit for bit (and adds 0 to moved); every centroid
 * that is recomputed or reseeded gets changed = 1 if its value differs in any
 * bit, else 0, which tells the next incremental assignment which centroids
 * moved. */
int skcq_finalize(int metric, float* sums, int32_t* counts, const int32_t* n_empty, int nblk, int k_pad, int bs,
                  const int32_t* k, int32_t* active, int32_t* converged, int32_t* iters_run, float* moved_hist,
                  int32_t* nempty_hist, int iter, float* C, uint8_t* changed, void* stream);

/* ---- incremental assignment ---------------------------------------------------
 * Exact: a centroid whose cluster kept its members keeps its value (see
 * skcq_finalize), so its scores are unchanged, and a point assigned to such a
 * centroid can only move to a centroid that moved. The host runs, per
 * iteration after the first: skcq_moved_lists; skcq_assign of every point
 * against the moved centroids only (gathered with skcq_gather_rows, labels
 * indexing the moved list); skcq_assign of the points whose centroid moved
 * (gathered) against all centroids; skcq_assign_merge. The labels equal a full
 * skcq_assign's. No counterpart in the reference, which rescans every
 * centroid each iteration (kmeans.py:136-149). */

/* changed[b][c] = 1 for every cluster c that gained or lost a point between
 * prev and labels (all = 1: every cluster, for the first assignment); rows of
 * problems with mask[b] == 0 are left as they are. */
int skcq_mark_changed(const int32_t* prev, const int32_t* labels, int nblk, int n_pad, int k_pad, const int32_t* n,
                      const int32_t* mask, int all, uint8_t* changed, void* stream);

/* For the problems with mask[b] != 0: mlist[b][0 .. mcount[b]) = the centroids
 * c < k[b] with changed[b][c], ascending; plist[b][0 .. pcount[b]) = the
 * points i < n[b] whose labels[b][i] has changed set, ascending. scratch:
 * skcq_moved_lists_scratch_bytes(nblk, n_pad, k_pad) bytes. */
size_t skcq_moved_lists_scratch_bytes(int nblk, int n_pad, int k_pad);
int skcq_moved_lists(const uint8_t* changed, const int32_t* labels, int nblk, int n_pad, int k_pad, const int32_t* n,
                     const int32_t* k, const int32_t* mask, int32_t* mlist, int32_t* mcount, int32_t* plist,
                     int32_t* pcount, void* scratch, size_t scratch_bytes, void* stream);

/* dst[b][j][:] = src[b][idx[b][j]][:] for j < count[b], 0 for count[b] <= j <
 * out_rows (src [nblk][src_rows][bs], idx row stride idx_ld). */
int skcq_gather_rows(const float* src, int src_rows, const int32_t* idx, int idx_ld, const int32_t* count, int nblk,
                     int out_rows, int bs, float* dst, void* stream);

/* In place on labels, for the active problems with a moved list: a point whose
 * centroid a did not move takes the best of mlist[b][0 .. mcount[b]) under
 * the reference formula (exact fp32 on CUDA cores, first maximum) when it
 * scores higher than a, or the same with a lower index. For short moved lists
 * (bs <= 32); replaces the tensor-core pass over the gathered moved centroids
 * and the first half of skcq_assign_merge (call that with zero mcount). */
int skcq_assign_moved_exact(int metric, const float* X, const float* C, const float* cnorm, int nblk, int n_pad,
                            int k_pad, int bs, const int32_t* n, const int32_t* active, const uint8_t* changed,
                            const int32_t* mlist, const int32_t* mcount, int32_t* labels, const float* C_old,
                            const float* cnorm_old, uint8_t* unres, void* stream);

/* Resolution of the points whose centroid moved (both entry points above and
 * below, when unres is not NULL): such a point takes the best moved centroid
 * when its score exceeds the point's score against a's value before the
 * update (C_old, cnorm_old: the centroids and norms that assignment used),
 * since that score bounds every unmoved centroid's unchanged score; otherwise
 * unres[b][i] = 1 and the point needs a search over all centroids (listed by
 * skcq_list_points). unres is written for every point. */

/* In place on labels (the previous assignment) for the active problems: a
 * point whose centroid a did not move (changed[b][a] == 0) takes
 * c = mlist[b][labels_m[b][i]] (the best moved centroid; labels_m from
 * skcq_assign against the gathered moved centroids) when c scores higher than
 * a under the reference formula, or the same with c < a; the points of plist
 * take labels_f[b][j] (skcq_assign of the gathered points, row stride p_pad).
 * labels_m[b][i] < 0 means point i was not scored against the moved
 * centroids (see skcq_mpass_points) and keeps its label. */
int skcq_assign_merge(int metric, const float* X, const float* C, const float* cnorm, int nblk, int n_pad, int k_pad,
                      int bs, const int32_t* n, const int32_t* active, const uint8_t* changed, const int32_t* mlist,
                      const int32_t* mcount, const int32_t* labels_m, const int32_t* plist, const int32_t* pcount,
                      int p_pad, const int32_t* labels_f, int32_t* labels, const float* C_old,
                      const float* cnorm_old, uint8_t* unres, void* stream);

/* Euclidean problems: flags[b][i] = 1 for the points the moved-centroid pass
 * must score -- those whose centroid moved and those not bit for bit equal to
 * their centroid (a point on its unmoved centroid has the largest score any
 * centroid can reach, so only an exact tie could move it). */
int skcq_mpass_points(const float* X, const float* C, const int32_t* labels, const uint8_t* changed,
                      const int32_t* n, const int32_t* active, int nblk, int n_pad, int k_pad, int bs,
                      uint8_t* flags, void* stream);

/* labels_m[b][list[b][j]] = sub[b][j] for j < count[b] (sub row stride s_pad,
 * list and labels_m row stride n_pad): results of a pass over a listed subset
 * back to point order. */
int skcq_scatter_sub(const int32_t* list, const int32_t* count, const int32_t* sub, int nblk, int s_pad, int n_pad,
                     int32_t* labels_m, void* stream);

/* plist[b][0 .. pcount[b]) = the points i < n[b] with flags[b][i] != 0,
 * ascending, for the problems with mask[b] != 0 (flags [nblk][n_pad]);
 * scratch: nblk * ceil(n_pad / 4096) ints. */
int skcq_list_points(const uint8_t* flags, int nblk, int n_pad, const int32_t* n, const int32_t* mask,
                     int32_t* plist, int32_t* pcount, void* scratch, size_t scratch_bytes, void* stream);

/* ---- codec post-processing ------------------------------------------------- */

/* Negative-scale flip of skcq/codebook/spherical.py:289-298: scale = <R, C[label]>;
 * flags[b] gets bit j set when some point with a negative scale has label j
 * (j < 63), and bit 63 when such a label is >= bs (the reference then raises
 * IndexError: it negates *columns* of the (k, d) centroid matrix). */
int skcq_flip_check(const float* R, const float* C, const int32_t* labels, int nblk, int n_pad, int k_pad, int bs,
                    const int32_t* n, uint64_t* flags, void* stream);
/* Negates dimension j of every centroid of problem b for each bit j set in
 * flags[b] (the reference's `centroids[:, neg_labels] = -centroids[:, neg_labels]`). */
int skcq_apply_flip(const uint64_t* flags, int nblk, int k_pad, int bs, float* C, void* stream);

/* idxs (n_blocks, n_rows) int64: labels of compacted points scattered back to
 * their source (row, block); unlisted (zero) points get label 0
 * (spherical.py:301-302, euclidean.py:500-501, shared reshape at :159 / :398). */
int skcq_scatter_labels(const int32_t* labels, const int32_t* rowmap, const int32_t* n, int nblk, int n_pad,
                        int shared, int n_rows, int n_blocks, int64_t* idxs, void* stream);

/* out[r] = 1 when ||W[r, :in_dim]|| < thr (the row zero mask of
 * aqlm.py:146-147 / spherical.py:150-151), else 0. */
int skcq_row_zero_mask(const float* W, int64_t ld, int n_rows, int in_dim, float thr, uint8_t* out, void* stream);

/* Spherical scales (spherical.py:178-184): scales[r][b] = <W[r, block b], C[idx]>,
 * 0 for rows flagged in row_zero. C is the fp32 centroid set (one problem when
 * shared). */
int skcq_spherical_scales(const float* W, int64_t ld, int n_rows, int bs, int n_blocks, int shared, const float* C,
                          int k_pad, const int64_t* idxs, const uint8_t* row_zero, float* scales, void* stream);

/* out[b][j][c] = bf16(C[b][c][j]) for c < K: the (n_blocks, bs, K) bf16
 * centroid tensor of spherical.py:176,188 / euclidean.py:415,419. */
int skcq_centroids_to_bf16(const float* C, int nblk, int k_pad, int bs, int K, uint16_t* out, void* stream);

/* out[r][c] = bf16(W[r][col0 + c]) (raw remainder, spherical.py:186). */
int skcq_copy_remainder(const float* W, int64_t ld, int n_rows, int col0, int rem, uint16_t* out, void* stream);

/* SSVQ fold (skcq/codebook/ssvq.py:43-53): s = sign(w) with 0 -> +1,
 * folded = w * s (f32), signs = s (int8), optional packed[r][w] bit (c%32) of
 * word c/32 set when s = -1. W is f32 (w_is_bf16 = 0) or bf16 bits. */
int skcq_ssvq_fold(const void* W, int w_is_bf16, int64_t ld, int n_rows, int in_dim, float* folded, int8_t* signs,
                   uint32_t* packed, void* stream);

/* Symmetric int<bits> fake quantisation of centroids, one scale per centroid
 * index over all blocks and dims (spherical.py:306-315, euclidean.py:186-195).
 * cb is the (rows = n_blocks*bs, K) bf16 tensor, updated in place. */
int skcq_quantize_centroids(uint16_t* cb, int rows, int K, int bits, void* stream);

/* int<bits> scale quantisation (spherical.py:57-69): q_scale = max|s|/levels,
 * q = clamp(rint(s / q_scale)); out is int8 (bits <= 8) or int16. q_scale is
 * written to *q_scale_out (device f32). When max|s| == 0 `out` is not written
 * and q_scale is 0, as in the reference. */
int skcq_quantize_scales(const float* scales, int64_t count, int bits, void* out, float* q_scale_out,
                         void* stream);

/* One codebook of a composite, as stored in its CWR (skcq/codebook/cwr.py). */
typedef struct skcq_codec_desc {
  int kind;              /* 0 spherical (scaled), 1 euclidean */
  int bs, n_blocks, K;   /* block size, blocks covered, centroids per block */
  int shared;            /* 1: one codebook for all blocks */
  const uint16_t* cent;  /* bf16 (shared ? 1 : n_blocks, bs, K) */
  const int64_t* idxs;   /* (n_blocks, idx_ld) */
  int64_t idx_ld;
  const void* scales;    /* (n_rows, scale_ld) or NULL */
  int scale_dtype;       /* 0 f32, 1 bf16, 2 f16, 3 int8, 4 int16 */
  float q_scale;         /* multiplier for int scales */
  int64_t scale_ld;
  const uint16_t* rem;   /* bf16 (n_rows, rem) or NULL */
  int rem_cols;
  const int8_t* signs;   /* int8 +-1 (n_rows, sign_ld) or NULL (SSVQ) */
  int sign_cols;         /* signed columns: min(in_dim, signs width) */
  int64_t sign_ld;
  /* Optional bf16 (shared ? 1 : n_blocks, K, bs) copy of cent with each
   * centroid's values contiguous (skcq_transpose_codebook), or NULL. When
   * given, the decode reads it: one memory sector per gathered centroid
   * instead of one per coordinate; the values are the same. */
  const uint16_t* cent_t;
} skcq_codec_desc;

#define SKCQ_MAX_CODECS 8

/* Composite decode (aqlm.py:137-141 over spherical.py:192-211,
 * euclidean.py:103-120, ssvq.py:57-66): out[r][c] = sum over codecs, in order,
 * of each codec's reconstruction; with raw != NULL, out = raw - that sum
 * (the AQLM residual target, aqlm.py:179/189). One streaming pass. */
int skcq_reconstruct(const skcq_codec_desc* codecs, int n_codecs, int n_rows, int in_dim, const float* raw,
                     int64_t raw_ld, float* out, int64_t out_ld, void* stream);

/* Least-squares primary scale re-fit (aqlm.py:147-179), in place on the f32
 * scales (n_rows, scale_ld) of `primary` (kind 0; signs honoured; its `scales`
 * field is ignored in favour of `scales`). recon is the full composite
 * reconstruction; rows flagged in row_zero get 0. */
int skcq_refit_scales(const skcq_codec_desc* primary, const float* raw, int64_t raw_ld, const float* recon,
                      int64_t recon_ld, int n_rows, const uint8_t* row_zero, float* scales, void* stream);

/* ---- codebook-expert forward (skcq/codebook_experts.py) -------------------- */

#define SKCQ_DTYPE_F32 0
#define SKCQ_DTYPE_BF16 1
#define SKCQ_DTYPE_F16 2
#define SKCQ_DTYPE_I8 3
#define SKCQ_DTYPE_I16 4

/* One codebook layer of a CodebookModule (_CodebookLayer, codebook_experts.py:77-150)
 * in the forward's device layout. Only the primary layer carries scales
 * (CodebookModule.forward applies p.scales only, codebook_experts.py:327-331). */
typedef struct skcq_fwd_layer {
  int n_blocks, bs, K;          /* bs <= 32, K <= 65536 */
  const void* table;            /* (n_blocks, K, bs) centroid vectors (skcq_transpose_codebook) */
  int table_dtype;              /* f32 | bf16 */
  const uint16_t* idx16;        /* (E, n_blocks, out) assignments (skcq_pack_indices16) */
  const void* scales;           /* (E, n_blocks, out) or NULL; f32 | bf16 | f16 | i8 | i16 */
  int scale_dtype;
  float q_scale;                /* multiplier for integer scales (scale_q_scale) */
  const void* remainder;        /* (E, out, rem), f32 | bf16 */
  int rem_dtype, rem;
  const uint32_t* sign_mask;    /* (E, n_blocks, out) bit j: column b*bs+j negated, or NULL */
  /* Per-token lookup table of this layer (the reference's matmul_gather
   * mode, codebook_experts.py:57-60), or NULL: lut[(b * K + k) * lut_tokens + t]
   * = <x_b(t), C_b[k]> for the lut_tokens rows t of x (skcq_lut_build). When
   * set, skcq_codebook_forward reads each block's dot from it instead of
   * gathering the centroid; the arithmetic is the same, so the output is
   * bit-identical. Requires sign_mask == NULL. */
  const float* lut;
  int lut_tokens;
} skcq_fwd_layer;

/* The lookup table of skcq_fwd_layer.lut for one layer: for every block b,
 * centroid k and row t < T of x (f32 | bf16, row stride x_ld),
 * lut[(b * K + k) * T + t] = sum over j in order of fma(x[t][b*bs + j],
 * C_b[k][j]) (the block dot the decode kernel forms; no signs).
 * lut holds n_blocks * K * T floats. */
int skcq_lut_build(const skcq_fwd_layer* layer, const void* x, int x_dtype, int64_t x_ld, int T, float* lut,
                   void* stream);

/* out[i] = (uint16) idx[i] for the reference's int64 assignments
 * (codebook_experts.py:95); an index outside [0, K) is stored as 0 and sets the
 * device error (the reference's gather raises). */
int skcq_pack_indices16(const int64_t* idx, int64_t n, int K, uint16_t* out, void* stream);

/* table[b][k][j] = codebook[b][j][k]: the reference's (n_blocks, bs, K) codebook
 * with each centroid's bs values made contiguous. dtype f32 | bf16. */
int skcq_transpose_codebook(const void* codebook, int dtype, int n_blocks, int bs, int K, void* table, void* stream);

/* mask[e][b][o] bit j = (signs[e][o][b*bs+j] < 0) for the int8 +-1 SSVQ signs
 * (codebook_experts.py:53-55); a sign other than +-1 sets the device error. */
int skcq_pack_sign_masks(const int8_t* signs, int E, int out, int64_t sign_ld, int n_blocks, int bs, uint32_t* mask,
                         void* stream);

/* Routing of CodebookExperts.forward (codebook_experts.py:462-470): pairs
 * p = kpos * T + token sorted stably by expert into perm[T*k]; seg[e] ..
 * seg[e+1] is expert e's run (seg has n_experts + 1 entries); row_of_pair[p]
 * is the inverse permutation; active[0] is the number of experts with rows and
 * active[1..] their ids ascending (n_experts + 1 entries). An expert id outside
 * [0, n_experts) sets the device error (the reference's one_hot raises),
 * except that with skip_negative != 0 a negative id marks a slot that is not
 * routed here (expert-parallel receive rows): such pairs sort after every
 * expert's run and are never computed. */
int skcq_route_sort(const int64_t* topk, int T, int k, int n_experts, int32_t* perm, int32_t* seg,
                    int32_t* row_of_pair, int32_t* active, void* scratch, size_t scratch_bytes, int skip_negative,
                    void* stream);

/* Scratch bytes with which skcq_route_sort spreads a large batch over many
 * CTAs (0: the one-CTA sort is used; it also runs when scratch is NULL or
 * smaller than this). The result is the same either way. */
size_t skcq_route_sort_scratch_bytes(int T, int k, int n_experts);

/* CodebookModule.forward over expert segments (codebook_experts.py:325-339):
 * for the rows r of segment s (expert seg_expert[s], or s when NULL; only the
 * segments listed in `active` when it is not NULL), input row
 * x[row_token[r] % T] (x[r] when row_token is NULL),
 *   part[split][r][o] = partial sum over the split's block range of
 *     sum_layers (scale * <x_b, signs * C_b[idx]>) + x_rem . rem_w (last split).
 * The sum over the n_split slots is the module output (skcq_sum_splits,
 * skcq_swiglu, skcq_combine). max_active bounds the active segments
 * (min(n_seg, rows) is always safe). rows_hint: expected rows per segment
 * (performance only; any segment length is computed correctly). part holds
 * n_split * P * out_dim floats. */
int skcq_codebook_forward(const skcq_fwd_layer* layers, int n_layers, const void* x, int x_dtype, int64_t x_ld,
                          const int32_t* row_token, int T, const int32_t* seg, const int32_t* seg_expert,
                          const int32_t* active, int n_seg, int max_active, int in_dim, int out_dim, int n_split,
                          int rows_hint, float* part, int64_t P, void* stream);

/* y[r][o] = sum over splits of part[split][r][o]; y f32 | bf16 with row stride y_ld. */
int skcq_sum_splits(const float* part, int n_split, int64_t P, int out_dim, void* y, int y_dtype, int64_t y_ld,
                    void* stream);

/* out = silu(sum_s gate[s]) * sum_s up[s] over n elements per split
 * (the SwiGLU of codebook_experts.py:427-433 with act_fn = SiLU). */
int skcq_swiglu(const float* gate, const float* up, int n_split, int64_t n, float* out, void* stream);

/* out[t] = sum over the token's k slots, in ascending (expert, kpos) order, of
 * (sum_s part[s][row_of_pair[kpos * T + t]]) * weights[t][kpos]
 * (codebook_experts.py:476-480); slots with a negative expert id are skipped.
 * part, weights and out f32 | bf16. */
int skcq_combine(const void* part, int part_dtype, int n_split, int64_t P, const int32_t* row_of_pair,
                 const int64_t* topk, const void* weights, int w_dtype, int T, int k, int H, void* out, int out_dtype,
                 void* stream);

/* ---- prefill forward on the tensor cores ------------------------------------
 * For large batches (many rows per expert) the active experts' weights are
 * decoded once into bf16 and multiplied on tcgen05 (kind::f16, fp32
 * accumulate). Operands live in the tcgen05 shared-memory image: A chunks of
 * 128 rows x 64 k (16 KB), W chunks of 256 outputs x 64 k (32 KB), K padded to
 * a multiple of 64 with zeros. KC = ceil(in_dim / 64), NT = ceil(out / 256).
 * Row tiles: 128 consecutive sorted rows of one expert. */

/* tiles[0] = number of row tiles; tile t = (row0, row1, slot) at
 * tiles[1 + 3t ..], slot = the expert's index in the active list of
 * skcq_route_sort. tiles holds 1 + 3 * max_tiles ints; max_tiles >=
 * ceil(rows / 128) + active experts. */
int skcq_prefill_plan(const int32_t* seg, int n_experts, int max_tiles, int32_t* tiles, void* stream);

/* A[t][kc] (max_tiles * KC * 16 KB, 16-byte aligned): mode 0, row r of tile t
 * is x[row_token[r] % T] (x[r] when row_token is NULL; x f32 | bf16); mode 1,
 * it is silu(x[r]) * up[r] (x and up f32: the SwiGLU of gate and up outputs).
 * Rows past a tile's end are zero. */
int skcq_prefill_pack(int mode, const void* x, int x_dtype, int64_t x_ld, const int32_t* row_token, int T,
                      const float* up, int64_t up_ld, int in_dim, const int32_t* tiles, int max_tiles, void* A,
                      void* stream);

/* W[slot][nt][kc] (max_slots * NT * KC * 32 KB, 16-byte aligned) for the
 * experts active[1 + slot] (slot < active[0]; expert = slot when active is
 * NULL): bf16 of sum over layers of (primary scale) * sign * centroid values
 * plus raw remainder columns, i.e. the module's dense expert weight
 * (codebook_experts.py:48-56, :325-339); block sizes up to 32. half = -1: tiles of
 * 256 outputs (NT = ceil(out / 256)); half = 0 | 1: tiles of 128 features
 * (NT = ceil(out / 128)) with this module's rows at [128 half, 128 half + 128)
 * of each 256-row chunk, so gate (0) and up (1) share one buffer. */
int skcq_prefill_dequant(const skcq_fwd_layer* layers, int n_layers, const int32_t* active, int max_slots,
                         int out_dim, int in_dim, int half, void* W, void* stream);

/* y[r][o] = sum_k A[r][k] * W_slot(r)[o][k] for the rows of every planned
 * tile (fp32 accumulation; y f32 | bf16, row stride y_ld; rows outside tiles
 * untouched). */
int skcq_prefill_gemm(const void* A, const void* W, const int32_t* tiles, int max_tiles, int in_dim, int out_dim,
                      void* y, int y_dtype, int64_t y_ld, void* stream);

/* Gate and up in one GEMM (W_gate_up from skcq_prefill_dequant with half 0 and
 * 1): for every planned tile, silu(x W_gate^T) * (x W_up^T) as bf16 rows in
 * the A image of the down projection (A_out: max_tiles * ceil(inter/64) *
 * 16 KB), zero past each tile's rows and past inter_dim (the SwiGLU of
 * codebook_experts.py:427-433 fused into the epilogue). */
int skcq_prefill_gemm_swiglu(const void* A, const void* W_gate_up, const int32_t* tiles, int max_tiles, int in_dim,
                             int inter_dim, void* A_out, void* stream);

/* ---- expert-parallel exchange over peer memory -------------------------------
 * CodebookExperts.forward (codebook_experts.py:454-481) with experts placed
 * across the GPUs of one node, one process per GPU. Rank r owns experts
 * [bounds[r], bounds[r + 1]) (bounds: world + 1 host ints, 0 .. n_experts).
 * Every rank allocates one exchange buffer laid out by skcq_ep_layout for the
 * same (world, capacity, top_k_cap, hidden) and maps the others' buffers
 * (skcq_ep_alloc / skcq_ep_open); `peers` is the host array of the world
 * buffers' addresses in this process (this rank's own at index rank).
 * capacity bounds the tokens any rank passes to one forward. Stores into a
 * peer's buffer are plain stores over NVLink; the caller orders the phases
 * across ranks with a stream-ordered barrier (a one-element all-reduce) after
 * skcq_ep_dispatch and after skcq_ep_return. */
#define SKCQ_EP_MAX_RANKS 8

/* Byte offsets in an exchange buffer: [0] token rows [world][capacity][hidden]
 * (4-byte slots), [1] slot ids and [2] slot weights [world][capacity][top_k_cap],
 * [3] row counts [8], [4] returned sums [world][capacity][hidden] (4-byte
 * slots), [5] total bytes. */
int skcq_ep_layout(int world, int capacity, int top_k_cap, int hidden, int64_t* offsets);

/* cudaMalloc'd, zeroed exchange buffer and its CUDA IPC handle (64 bytes). */
int skcq_ep_alloc(size_t bytes, void** ptr, void* ipc_handle);
/* Map another process's buffer (peer access enabled on first use). */
int skcq_ep_open(const void* ipc_handle, void** ptr);
int skcq_ep_close(void* ptr);
int skcq_ep_free(void* ptr);

/* Send this rank's T tokens: x (T, hidden) f32 | bf16 with row stride x_ld,
 * topk (T, k) int64 global expert ids, weights (T, k) f32 | bf16. Every row is
 * stored once into each rank that owns one of its experts, with per slot the
 * local expert id there (-1 when owned elsewhere) and the weight; pos (T x
 * world ints) receives each token's row index at each rank (-1: not sent), and
 * every rank's count of rows from this rank is published. chunk_counts:
 * device scratch of 8 * max(1, ceil(T / 1024)) ints. An id outside
 * [0, n_experts) sets the device error and is not routed. */
int skcq_ep_dispatch(const void* x, int x_dtype, int64_t x_ld, const int64_t* topk, const void* weights, int w_dtype,
                     int T, int k, int n_experts, const int32_t* bounds, void* const* peers, int world, int rank,
                     int capacity, int top_k_cap, int hidden, int32_t* chunk_counts, int32_t* pos, void* stream);

/* The rows received in this rank's buffer as a routing of its local experts:
 * topk_out / weights_out (world * capacity, k) int64 / f32, id -1 (weight 0)
 * for slots owned elsewhere and rows past a source's count (feed
 * skcq_route_sort with skip_negative = 1). */
int skcq_ep_unpack(const void* buffer, int world, int capacity, int k, int top_k_cap, int hidden, int64_t* topk_out,
                   float* weights_out, void* stream);

/* For every received row r = s * capacity + i (i below source s's count):
 * sum over its local slots, in ascending (expert, slot) order, of
 * (sum_split part[split][row_of_pair[kpos * world * capacity + r]]) * weight,
 * stored in out_dtype into rank s's returned sums at [rank][i] (the combine of
 * codebook_experts.py:476-480, restricted to this rank's experts, written
 * straight into the source's memory). P = world * capacity * k. */
int skcq_ep_return(const void* part, int part_dtype, int n_split, int64_t P, const int32_t* row_of_pair,
                   const int64_t* topk_local, const float* weights_local, const void* buffer, void* const* peers,
                   const int32_t* bounds, int n_experts, int world, int rank, int capacity, int k, int top_k_cap,
                   int hidden, int out_dtype, void* stream);

/* out[t] = sum over ranks d ascending with pos[t][d] >= 0 of the sum rank d
 * returned for token t (ret_dtype), stored as out_dtype (T, hidden). */
int skcq_ep_gather(const void* buffer, const int32_t* pos, int T, int world, int capacity, int top_k_cap, int hidden,
                   int ret_dtype, void* out, int out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SKCQ_B200_H */
