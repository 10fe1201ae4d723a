/*
 * mpo_b200.h -- C ABI of libmpo_b200.so, the sm_100a (B200) kernels behind
 * the point-cloud hot path of gamzerA/mps-pointops v1.0.0.
 *
 * Conventions (every entry point):
 *   - Pointers are CUDA device pointers to dense row-major arrays on the
 *     current device; shapes are given by the int64 sizes.  float = IEEE
 *     binary32.  Nullable pointers say so.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Every call
 *     only enqueues work and returns; results are ready when the stream is.
 *   - Outputs and workspaces are owned by the caller.  Every output slot is
 *     written, padding included.  Nothing is allocated inside the library,
 *     except the exchange arrays of mpo_p2p_slots_create (device memory
 *     that other processes map through CUDA IPC).
 *     Workspaces must be 256-byte aligned (as cudaMalloc returns them;
 *     MPO_ERR_INVALID_ARGUMENT otherwise).  Float arrays need only 4-byte
 *     alignment: kernels use 16-byte vector loads on a caller's array only
 *     when its base address allows them.
 *   - The return value is 0 (MPO_OK) or an MPO_ERR_* code; mpo_last_error()
 *     then holds a message (per calling thread).
 *   - Squared distances are ((d0*d0 + d1*d1) + d2*d2) for D == 3 and the
 *     sequential sum for D != 3, d = a - b, each operation rounded on its own
 *     (no FMA), exactly as the reference's CPU code; ties go to the lowest
 *     index.
 *
 * Each declaration cites the reference interface it replaces (paths relative
 * to the reference project).  The reference dispatches to Metal through
 * torch.mps.compile_shader (mps_pointops/ops.py:33-37); these entry points
 * take the place of those `library.<kernel>(...)` calls.
 */
#ifndef MPO_B200_H_
#define MPO_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MPO_API __attribute__((visibility("default")))
#else
#define MPO_API
#endif

#define MPO_ABI_VERSION 9

#define MPO_OK 0
#define MPO_ERR_INVALID_ARGUMENT 1
#define MPO_ERR_CUDA 2
#define MPO_ERR_UNSUPPORTED 3
#define MPO_ERR_WORKSPACE_TOO_SMALL 4

/* ABI version of the loaded library (MPO_ABI_VERSION). */
MPO_API int32_t mpo_abi_version(void);

/* Message of the last failed call on this host thread ("" if none). */
MPO_API const char* mpo_last_error(void);

/* Number of kernels this library has launched in the process (all devices,
 * all threads).  No counterpart in the reference; used to count the native
 * launches inside a timed region. */
MPO_API uint64_t mpo_launch_count(void);

/* MPO_OK if `device` is an sm_100 part this build runs on, else
 * MPO_ERR_UNSUPPORTED.  Replaces the Metal runtime probes
 * mps_pointops/_ball_query_mps.py:34-63 (_require_compile_shader,
 * _check_simd_width). */
MPO_API int mpo_device_supported(int device);

/* ------------------------------------------------------------------ FPS
 * Replaces the `furthest_point_sample` and `fps_update_partials` /
 * `fps_reduce_partials` dispatches of mps_pointops/ops.py:53-141
 * (kernels fps.metal:19-107, fps_multigroup.metal:10-133); contract of
 * mps_pointops/reference.py:27-58.
 *   xyz (B,N,3) -> out (B,npoint), int64 or, with out_int32 != 0, int32
 *   (the pointnet2_ops form of mps_pointops/compat.py:53-59).
 *   skip_near_origin: points with ((x*x+y*y)+z*z) < fl32(1e-3) are never
 *   picked after the start.  Requires N >= 1 when npoint > 0 and
 *   0 <= start_idx < N.  strategy mirrors the reference's `strategy=`
 *   argument: MPO_FPS_AUTO picks by size, MPO_FPS_SINGLE runs one CTA per
 *   cloud (N <= 8192), MPO_FPS_GROUP spreads each cloud over a cooperative
 *   group of CTAs (the large-cloud path, selectable at any size).  Any
 *   N < 2^31 is accepted: above 8192 points per SM every SM takes part and
 *   each CTA keeps its extra points in shared memory and then in the
 *   workspace.  The workspace (mpo_fps_workspace_bytes) holds the cross-CTA
 *   step slots of the group path and that overflow tier (16 bytes per point
 *   beyond 22,528 per SM); status_out (nullable, device int32) receives 0,
 *   or 1 if a bounded cross-CTA wait gave up. */
#define MPO_FPS_AUTO 0
#define MPO_FPS_SINGLE 1
#define MPO_FPS_GROUP 2
MPO_API size_t mpo_fps_workspace_bytes(int64_t B, int64_t N, int64_t npoint, int strategy);
MPO_API int mpo_fps(const float* xyz, int64_t B, int64_t N, int64_t npoint, int64_t start_idx,
                    int skip_near_origin, int out_int32, int strategy, void* out,
                    int32_t* status_out, void* workspace, size_t workspace_bytes, void* stream);

/* mpo_fps plus the fused gather of the sampled points: out_xyz (B, npoint, 3)
 * receives xyz[b, out[b, i], :] -- the FPS -> gather_operation step of a
 * PointNet++ set abstraction (mps_pointops/compat.py:53-65;
 * tests/test_pointnet2_e2e.py:37-39) without a separate launch.  Same
 * arguments, workspace and status as mpo_fps; out_xyz may be NULL. */
MPO_API int mpo_fps_gather(const float* xyz, int64_t B, int64_t N, int64_t npoint,
                           int64_t start_idx, int skip_near_origin, int out_int32, int strategy,
                           void* out, float* out_xyz, int32_t* status_out, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Allocation-free FPS.  No counterpart in the reference: it exists for
 * callers that cannot allocate device memory (for example a plugin given only
 * its input and output buffers), so it takes no workspace.  Same contract,
 * arguments and results as mpo_fps; the CTA-group path keeps its step slots
 * in a fixed 40 KiB array inside the library (per device) -- enough for any
 * batch on a 148-SM B200, since cooperative waves reuse the slots; a launch
 * that would need more, or a cloud above 22,528 points per SM (3,334,144 on
 * a 148-SM B200, whose extra points would need workspace), is rejected with
 * MPO_ERR_INVALID_ARGUMENT.  The first call on a device (and the first after
 * the device's context is replaced, e.g. by cudaDeviceReset) looks the array
 * up with cudaGetSymbolAddress and should come before any stream capture;
 * any number of devices is served.  All calls share the array: calls whose
 * GPU work overlaps race on it. */
MPO_API int mpo_fps_noalloc(const float* xyz, int64_t B, int64_t N, int64_t npoint,
                            int64_t start_idx, int skip_near_origin, int out_int32, int strategy,
                            void* out, int32_t* status_out, void* stream);

/* ------------------------------------------------------------------ kNN
 * Replaces the `knn` (D == 3, kernels/knn.metal:32-140) and
 * `feature_knn_dense` (D != 3, kernels/feature_knn.metal:51-164) dispatches
 * of mps_pointops/ops.py:144-205.
 *   query (B,M,D), ref (B,N,D) -> dist (B,M,k) Euclidean (sqrt after
 *   selection), idx (B,M,k) int64, sorted by (squared distance, index).
 *   sqdist (nullable, (B,M,k)) receives the squared distances before the
 *   square root.  1 <= k <= min(N, 256).  D == 3 drops NaN candidates and
 *   ranks +inf; D != 3 drops every non-finite candidate; unfilled slots are
 *   (inf, -1).
 *   workspace: mpo_knn_workspace_bytes(B, M, N, D, k) bytes of device memory
 *   (0 when the call needs none: D == 3, small or narrow problems).  Feature
 *   kNN with 16 <= D <= 96, k <= 32 and N >= 2048 proposes candidates with
 *   tensor-core (tcgen05) scores and ranks them by the exact fp32 SD. */
MPO_API size_t mpo_knn_workspace_bytes(int64_t B, int64_t M, int64_t N, int64_t D, int64_t k);
MPO_API int mpo_knn(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int64_t D,
            int64_t k, float* dist, int64_t* idx, float* sqdist, void* workspace,
            size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ ball query
 * Replaces the `ball_query_f32` dispatch of mps_pointops/_ball_query_mps.py:
 * 122-166 (kernels/ball_query.metal:30-124) behind ops.ball_query
 * (mps_pointops/ops.py:208-227); contract of mps_pointops/reference.py:83-121.
 *   query (B,M,3), ref (B,N,3), radius_sq = fl32(fl32(r)*fl32(r)) ->
 *   dist2 (B,M,K) f32 and idx (B,M,K) int64: the first K reference points in
 *   input order with squared distance < radius_sq; empty slots (-1, 0).
 *   query_lengths / ref_lengths (nullable, (B,) int64): queries at or beyond
 *   query_lengths[b] are all padding, references at or beyond ref_lengths[b]
 *   never match (mps_pointops/_ball_query_mps.py:73-84). */
MPO_API int mpo_ball_query(const float* query, const float* ref, const int64_t* query_lengths,
                   const int64_t* ref_lengths, int64_t B, int64_t M, int64_t N, int64_t K,
                   float radius_sq, float* dist2, int64_t* idx, void* stream);

/* pointnet2_ops form (mps_pointops/compat.py:76-85): xyz (B,N,3), new_xyz
 * (B,npoint,3) -> idx (B,npoint,nsample) int32 where an empty slot repeats
 * the query's first hit, and a query without hits is all zeros. */
MPO_API int mpo_ball_query_pointnet2(const float* xyz, const float* new_xyz, int64_t B, int64_t N,
                             int64_t npoint, int64_t nsample, float radius_sq, int32_t* idx,
                             void* stream);

/* Backward of the squared distances (mps_pointops/_ball_query_mps.py:168-203):
 * grad_query[b,m] = sum_s 2 g (q - x_idx), grad_ref[b,idx] -= 2 g (q - x_idx)
 * over the slots with idx >= 0.  grad_query and grad_ref (nullable) are
 * overwritten. */
MPO_API int mpo_ball_query_backward(const float* grad_dist2, const float* query, const float* ref,
                            const int64_t* idx, int64_t B, int64_t M, int64_t N, int64_t K,
                            float* grad_query, float* grad_ref, void* stream);

/* ------------------------------------------------------------------ PointNet++ propagation
 * Replaces `three_nn_f32` (kernels/pointnet2.metal:8-50) behind
 * mps_pointops/pointnet2.py:75-100; contract of pointnet2.py:54-72.
 *   unknown (B,N,3), known (B,M,3), M >= 3 -> dist (B,N,3) Euclidean,
 *   idx (B,N,3) int32, ordered by (squared distance, index) with NaN last. */
MPO_API int mpo_three_nn(const float* unknown, const float* known, int64_t B, int64_t N, int64_t M,
                 float* dist, int32_t* idx, void* stream);

/* Replaces `three_interpolate_f32` (kernels/pointnet2.metal:52-71) behind
 * mps_pointops/pointnet2.py:150-166; contract of pointnet2.py:135-147.
 *   features (B,C,M), idx (B,N,3) int32 in [0,M), weights (B,N,3) ->
 *   out (B,C,N) = ((f0*w0 + f1*w1) + f2*w2). */
MPO_API int mpo_three_interpolate(const float* features, const int32_t* idx, const float* weights,
                          int64_t B, int64_t C, int64_t M, int64_t N, float* out, void* stream);

/* Replaces `three_interpolate_backward_f32` (kernels/pointnet2.metal:76-103)
 * behind mps_pointops/pointnet2.py:168-188: grad_features (B,C,M) is
 * overwritten with sum over (n,t) of grad_out[b,c,n] * weights[b,n,t] at
 * idx[b,n,t]. */
MPO_API int mpo_three_interpolate_backward(const float* grad_out, const int32_t* idx,
                                   const float* weights, int64_t B, int64_t C, int64_t M,
                                   int64_t N, float* grad_features, void* stream);

/* Replaces the host bounds check of mps_pointops/pointnet2.py:130-131
 * (torch.any((indices < 0) | (indices >= M)).item()): *flag (int32, device)
 * becomes 1 if any of the n indices (int32, or int64 when idx_is_int64) lies
 * outside [0, upper), else 0.  Asynchronous: the caller reads the flag after
 * queueing the interpolation (whose kernels skip out-of-range indices) and
 * raises then. */
MPO_API int mpo_index_check(const void* idx, int idx_is_int64, int64_t n, int64_t upper,
                            int32_t* flag, void* stream);

/* ------------------------------------------------------------------ Chamfer
 * Replaces `chamfer_nearest_f32` / `chamfer_nearest_nd_f32`
 * (kernels/chamfer_nn.metal:13-82, 159-226) behind
 * mps_pointops/chamfer.py:122-158; contract of chamfer.py:161-212 and
 * 297-308 (squared L2).
 *   x (B,P,D), y (B,Q,D), lengths (nullable, (B,) int64) ->
 *   idx_x (B,P): the first y index with the smallest squared distance among
 *   y[:y_lengths[b]] (the first valid y even if every distance overflows to
 *   +inf), -1 for padded x rows or an empty y cloud; dist_x (B,P) its squared
 *   distance, 0 where idx_x is -1.  With bidirectional != 0 the same is
 *   computed for y against x into dist_y / idx_y from the same pair
 *   evaluations.  The workspace (mpo_chamfer_workspace_bytes) holds the
 *   partial column minima. */
MPO_API size_t mpo_chamfer_workspace_bytes(int64_t B, int64_t P, int64_t Q, int64_t D,
                                   int bidirectional);
MPO_API int mpo_chamfer_nearest(const float* x, const float* y, const int64_t* x_lengths,
                        const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q, int64_t D,
                        int bidirectional, float* dist_x, int64_t* idx_x, float* dist_y,
                        int64_t* idx_y, void* workspace, size_t workspace_bytes, void* stream);

/* Backward of the selected squared distances (mps_pointops/chamfer.py:215-251)
 * for one or both directions: for every x row with idx_x >= 0,
 *   g = 2 * grad_dist_x * (x - y[idx_x]);  grad_x += g;  grad_y[idx_x] -= g
 * and symmetrically for y rows when grad_dist_y is non-NULL.  grad_x and
 * grad_y are overwritten. */
MPO_API int mpo_chamfer_backward(const float* x, const float* y, int64_t B, int64_t P, int64_t Q,
                         int64_t D, const int64_t* idx_x, const float* grad_dist_x,
                         const int64_t* idx_y, const float* grad_dist_y, float* grad_x,
                         float* grad_y, void* stream);

/* L1 Chamfer (norm=1): replaces chamfer_nearest_l1_f32 (kernels/chamfer_nn.metal:86-152)
 * and the CPU path of mps_pointops/chamfer.py:161-212 with norm == 1.  Same
 * arguments and conventions as mpo_chamfer_nearest without a workspace: the
 * distance is |d0| + |d1| + ... in dimension order (d = query - ref, each
 * operation rounded on its own), first minimum with the lowest index on
 * ties; invalid rows get (0, -1).  Both directions with D == 3 and P, Q >= 512
 * run the symmetric tile kernel, which needs scratch: it uses idx_x, idx_y
 * and the first word of dist_x during the call (all of them are overwritten
 * with the results).  On that path the four outputs must not overlap each
 * other or the inputs, and idx_x / idx_y must be 8-byte aligned (both are
 * checked: MPO_ERR_INVALID_ARGUMENT). */
MPO_API int mpo_chamfer_nearest_l1(const float* x, const float* y, const int64_t* x_lengths,
                                   const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q,
                                   int64_t D, int bidirectional, float* dist_x, int64_t* idx_x,
                                   float* dist_y, int64_t* idx_y, void* stream);
/* Its backward (mps_pointops/chamfer.py:269-293, PyTorch3D's subgradient): for
 * every x row with idx_x >= 0, g = s * grad_dist_x with s = +1 where
 * x > y[idx_x] and -1 otherwise (equality included); grad_x += g;
 * grad_y[idx_x] -= g; symmetrically for y.  Outputs overwritten. */
MPO_API int mpo_chamfer_l1_backward(const float* x, const float* y, int64_t B, int64_t P,
                                    int64_t Q, int64_t D, const int64_t* idx_x,
                                    const float* grad_dist_x, const int64_t* idx_y,
                                    const float* grad_dist_y, float* grad_x, float* grad_y,
                                    void* stream);

/* float64 Chamfer search: the reference accepts float64 on every device but
 * MPS (mps_pointops/chamfer.py:101-102, docstring :365) and computes it with
 * its tiled torch search (chamfer.py:161-212); this replaces that search for
 * float64 CUDA tensors.  Same arguments and conventions as
 * mpo_chamfer_nearest (norm 2: squared L2; norm 1: L1) with double inputs
 * and distances, all arithmetic in double with every operation rounded, in
 * dimension order; first minimum, lowest index on ties; invalid rows get
 * (0, -1).  No workspace. */
MPO_API int mpo_chamfer_nearest_f64(const double* x, const double* y, const int64_t* x_lengths,
                                    const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q,
                                    int64_t D, int norm, int bidirectional, double* dist_x,
                                    int64_t* idx_x, double* dist_y, int64_t* idx_y, void* stream);
/* Its backward (mps_pointops/chamfer.py:227-251 for norm 2, 269-293 for
 * norm 1), in double: as mpo_chamfer_backward / mpo_chamfer_l1_backward.
 * Outputs overwritten. */
MPO_API int mpo_chamfer_backward_f64(const double* x, const double* y, int64_t B, int64_t P,
                                     int64_t Q, int64_t D, int norm, const int64_t* idx_x,
                                     const double* grad_dist_x, const int64_t* idx_y,
                                     const double* grad_dist_y, double* grad_x, double* grad_y,
                                     void* stream);

/* Fused loss for chamfer_distance with the common reductions and no weights
 * or normals (mps_pointops/chamfer.py:436-488, PyTorch3D conventions):
 * the search of mpo_chamfer_nearest (same dist/idx outputs), then
 *   per cloud  r_b = red(dist_x[b, :x_len]) (+ red(dist_y[b, :y_len]) when
 *              bidirectional), red = sum (point_mode 0) or mean over the
 *              valid points, empty -> divide by 1 (point_mode 1);
 *   loss       r (batch_mode 0, (B,) floats), sum_b r_b (1) or its mean (2).
 * Sums run in a fixed order (bit-reproducible).  Workspace:
 * mpo_chamfer_loss_workspace_bytes.  No reference counterpart as a single
 * call: it replaces the search plus the torch reductions of chamfer.py. */
MPO_API size_t mpo_chamfer_loss_workspace_bytes(int64_t B, int64_t P, int64_t Q, int64_t D,
                                                int bidirectional);
MPO_API int mpo_chamfer_loss(const float* x, const float* y, const int64_t* x_lengths,
                             const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q,
                             int64_t D, int bidirectional, int point_mode, int batch_mode,
                             float* dist_x, int64_t* idx_x, float* dist_y, int64_t* idx_y,
                             float* loss, void* workspace, size_t workspace_bytes, void* stream);
/* Gradient of mpo_chamfer_loss: grad_loss is the loss gradient ((B,) for
 * batch_mode 0, one float otherwise); grad_x and grad_y are overwritten with
 * the sums of 2 c (q - r[idx]) over the matched pairs, c = the chain-rule
 * coefficient of each valid point's distance. */
MPO_API int mpo_chamfer_loss_backward(const float* x, const float* y, const int64_t* x_lengths,
                                      const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q,
                                      int64_t D, int bidirectional, int point_mode, int batch_mode,
                                      const int64_t* idx_x, const int64_t* idx_y,
                                      const float* grad_loss, float* grad_x, float* grad_y,
                                      void* stream);

/* Input checks of mps_pointops/chamfer.py:79-110 in one launch: flags
 * (device int32[4]) receive {x has a non-finite valid coordinate, the same
 * for y, x_lengths outside [0,P], y_lengths outside [0,Q]}, each 0 or 1. */
MPO_API int mpo_chamfer_check_inputs(const float* x, const float* y, const int64_t* x_lengths,
                                     const int64_t* y_lengths, int64_t B, int64_t P, int64_t Q,
                                     int64_t D, int32_t* flags, void* stream);

/* ------------------------------------------------------------------ SA grouping
 * gather_operation / grouping_operation of pointnet2_ops, which the reference
 * serves with torch gather (mps_pointops/compat.py:62-73):
 *   out[b, c, p, s] = features[b, c, idx[b, p, s]]      features (B, C, N),
 *   idx (B, P, S) int32 (idx_is_int64 = 0) or int64, out (B, C, P, S); gather
 *   is S = 1.  Indices outside [0, N) give 0 (check them with
 *   mpo_index_check, as the reference's gather raises on them).
 * The backward overwrites grad_features (B, C, N) with the scatter-add of
 * grad_out over idx (float atomics: the order of additions into one element
 * is not fixed).
 * Workspace (optional, 16-byte aligned): when every point is gathered several
 * times (P * S >= N, C >= 4), mpo_group_points_workspace_bytes() > 0 and a
 * workspace of that size lets both calls work on a (B, N, C) copy of the
 * features or gradient, so that a point's channels are contiguous and every
 * global access is coalesced; with NULL or too small a workspace they work on
 * (B, C, N) directly (same forward bits; the backward's float additions may
 * come in another order). */
MPO_API size_t mpo_group_points_workspace_bytes(int64_t B, int64_t C, int64_t N, int64_t P,
                                                int64_t S);
MPO_API int mpo_group_points(const float* features, const void* idx, int idx_is_int64,
                             int64_t B, int64_t C, int64_t N, int64_t P, int64_t S, float* out,
                             void* workspace, size_t workspace_bytes, void* stream);
/* Gradient of the points gathered by mpo_fps_gather: grad_xyz (B,N,3) is
 * overwritten with the scatter-add of grad (B,P,3) over idx (B,P) int32
 * (float atomics) -- the backward of gather_operation on the coordinates. */
MPO_API int mpo_gather_points_backward(const float* grad, const int32_t* idx, int64_t B,
                                       int64_t N, int64_t P, float* grad_xyz, void* stream);
MPO_API int mpo_group_points_backward(const float* grad_out, const void* idx, int idx_is_int64,
                                      int64_t B, int64_t C, int64_t N, int64_t P, int64_t S,
                                      float* grad_features, void* workspace,
                                      size_t workspace_bytes, void* stream);

/* Fused set-abstraction grouping: the composition of
 * tests/test_pointnet2_e2e.py:40-44 (compat.ball_query, grouping of xyz minus
 * the centre, grouping of the features, concatenation along channels) in two
 * launches and without temporaries.  xyz (B,N,3), new_xyz (B,P,3), features
 * (B,C,N) (C may be 0), radius_sq = fl32(fl32(r)^2).  Writes idx (B,P,S)
 * int32 -- the pointnet2_ops ball query of mpo_ball_query_pointnet2 -- and
 * out (B, 3*use_xyz + C, P, S): channels 0..2 = xyz[b, idx, :] - new_xyz[b, p, :]
 * when use_xyz != 0, then the grouped features.  The optional workspace
 * (mpo_query_and_group_workspace_bytes) plays the same role as in
 * mpo_group_points. */
MPO_API size_t mpo_query_and_group_workspace_bytes(int64_t B, int64_t N, int64_t P, int64_t S,
                                                   int64_t C);
MPO_API int mpo_query_and_group(const float* xyz, const float* new_xyz, const float* features,
                                int64_t B, int64_t N, int64_t P, int64_t S, int64_t C,
                                float radius_sq, int use_xyz, int32_t* idx, float* out,
                                void* workspace, size_t workspace_bytes, void* stream);
/* Its backward: grad_xyz (B,N,3) and grad_features (B,C,N) receive the
 * scatter-add of grad_out over idx (float atomics), grad_new_xyz (B,P,3) minus
 * the slot sum of the coordinate channels (slot order); each output is
 * nullable and, when given, overwritten.  Workspace as for the forward. */
MPO_API int mpo_query_and_group_backward(const float* grad_out, const int32_t* idx, int64_t B,
                                         int64_t N, int64_t P, int64_t S, int64_t C,
                                         int use_xyz, float* grad_xyz, float* grad_new_xyz,
                                         float* grad_features, void* workspace,
                                         size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ spatial grid
 * Grid-accelerated exact search over one cloud: replaces the reference's
 * opt-in spatial index (mps_pointops/spatial.py:76-264, SpatialIndex with
 * its Morton BVH, kernels spatial_bvh.metal / spatial_keys.metal).  Results
 * equal the brute-force searches' (mpo_knn D == 3 policy; mpo_ball_query).
 * A uniform grid of dims[0] x dims[1] x dims[2] cubic cells of side
 * cell_size from origin (both HOST arrays of 3) is built by counting sort:
 * cell_start (device int32, cells + 1 entries), sorted_points (device, N
 * float4 = x, y, z, original index bits), extra_points (device, room for N
 * float4: the points with a non-finite coordinate) and *n_extra_out (device
 * int32: their count).  Points outside the box are clamped into the edge
 * cells.  sorted_points and extra_points must be 16-byte aligned.
 * Workspace: mpo_grid_workspace_bytes(N, cells). */
MPO_API size_t mpo_grid_workspace_bytes(int64_t N, int64_t cells);
MPO_API int mpo_grid_build(const float* points, int64_t N, const float* origin, float cell_size,
                           const int* dims, int* cell_start, float* sorted_points,
                           float* extra_points, int32_t* n_extra_out, void* workspace,
                           size_t workspace_bytes, void* stream);
/* k nearest (k <= 32) of Q queries (Q, 3): dist (Q, k) Euclidean, idx (Q, k)
 * int64 original indices, ascending (squared distance, index), NaN dropped,
 * (inf, -1) padding.  n_extra: the host copy of the build's count. */
MPO_API int mpo_grid_knn(const float* query, int64_t Q, const float* origin, float cell_size,
                         const int* dims, const int* cell_start, const float* sorted_points,
                         const float* extra_points, int32_t n_extra, int64_t k, float* dist,
                         int64_t* idx, void* stream);
/* First K (<= 32) points in input order with squared distance < radius_sq:
 * dist2 (Q, K), idx (Q, K) int64, (0, -1) padding.  radius is the float32
 * radius (it sets how many cells around the query are searched). */
MPO_API int mpo_grid_ball_query(const float* query, int64_t Q, const float* origin,
                                float cell_size, const int* dims, const int* cell_start,
                                const float* sorted_points, float radius, float radius_sq,
                                int64_t K, float* dist2, int64_t* idx, void* stream);

/* ------------------------------------------------------------------ flat batches
 * The torch_cluster-style API of mps_pointops/flat.py:161-425 works on flat
 * (ragged) batches: x (nx, D) reference rows and y (ny, D) query rows, sorted
 * by cloud, with int64 offset arrays ptr_x and ptr_y of `segments + 1`
 * entries (ptr[b] = first row of cloud b, ptr[segments] = the row count;
 * flat.py:67-97).  Results are GLOBAL row numbers of x.  `status` (device
 * int32, required) is zeroed by the call and then set to 1 when the offset
 * arrays do not run from 0 to the row counts without decreasing (the checks
 * of mps_pointops/_flat_search_mps.py:41-63); the search then writes nothing.
 *
 * kNN: replaces knn_indices (mps_pointops/_flat_search_mps.py:79-108,
 * kernels flat_search.metal:45-150 and feature_knn.metal:166-199); contract
 * of the CPU path flat.py:264-288 (_reference_search): out (ny, k) holds the
 * k nearest rows of each query's cloud in ascending (squared distance, index)
 * order, non-finite distances dropped, -1 padding.  k <= 256.
 * max_segment_x: the longest reference cloud (an upper bound is allowed; it
 * selects the kernel). */
MPO_API int mpo_flat_knn(const float* x, const float* y, const int64_t* ptr_x,
                         const int64_t* ptr_y, int64_t segments, int64_t nx, int64_t ny,
                         int64_t D, int64_t k, int64_t max_segment_x, int64_t* out,
                         int32_t* status, void* stream);

/* Radius: replaces radius_indices (mps_pointops/_flat_search_mps.py:111-147,
 * kernel flat_search.metal:172-276); contract of flat.py:264-288: out
 * (ny, max_neighbors) holds the first max_neighbors rows of the query's cloud
 * IN INPUT ORDER whose squared distance is < radius_sq, -1 padding.  D = 3.
 * radius_sq = fl32(r * r) with r * r in double (_flat_search_mps.py:66-76).
 * ignore_same_index != 0 skips the x row whose global number equals the
 * query's, before the cap (pyg-lib's radius; mps_pointops/pyg.py:100-126). */
MPO_API int mpo_flat_radius(const float* x, const float* y, const int64_t* ptr_x,
                            const int64_t* ptr_y, int64_t segments, int64_t nx, int64_t ny,
                            float radius_sq, int64_t max_neighbors, int ignore_same_index,
                            int64_t* out, int32_t* status, void* stream);

/* FPS: replaces fps_flat (mps_pointops/_flat_fps_mps.py:35-96, kernel
 * fps_flat.metal); contract of flat.py:161-217 with the per-cloud sampling of
 * mps_pointops/reference.py:27-58.  Cloud b (rows ptr[b] .. ptr[b+1] of x,
 * D = 3) yields out_ptr[b+1] - out_ptr[b] samples into out[out_ptr[b] ..],
 * as global rows, starting from the LOCAL index starts[b] (device int64).
 * total_out = out_ptr[segments]; max_len = the longest cloud (exact or an
 * upper bound; clouds above 8192 points use the cooperative CTA-group path
 * and need mpo_flat_fps_workspace_bytes(segments, max_len) of workspace).
 * status: 0, 1 (a group exchange timed out), or 2 (a cloud with samples is
 * empty, longer than max_len, or its start is out of range: the checks of
 * _flat_fps_mps.py:67-80; that cloud's samples are not written). */
MPO_API size_t mpo_flat_fps_workspace_bytes(int64_t segments, int64_t max_len);
MPO_API int mpo_flat_fps(const float* x, const int64_t* ptr, const int64_t* out_ptr,
                         const int64_t* starts, int64_t segments, int64_t total_n,
                         int64_t total_out, int64_t max_len, int64_t* out, int32_t* status,
                         void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ row gathers
 * Neighbour gathers with -1 padding: replaces the `_gather_neighbors` tensor
 * code of the PyTorch3D adapter (mps_pointops/pytorch3d.py:26-38, `knn` of
 * ball_query with return_nn) and the gathers of Pointcept's `grouping`
 * (mps_pointops/pointcept.py:168-203).
 *   src (B, N, W) float32 rows, idx (B, R) int64 (idx_int32 == 0) or int32:
 *   out[(b R + r) * out_stride + out_offset + w] = src[b, idx[b, r], w], or 0
 *   when the index is outside [0, N).  centers (nullable, (B R / K, W)):
 *   subtract centers[(b R + r) / K, w] from valid rows (the relative
 *   coordinates of `grouping(with_xyz=True)`).  No workspace. */
MPO_API int mpo_gather_rows(const float* src, int64_t B, int64_t N, int64_t W, const void* idx,
                            int idx_int32, int64_t R, const float* centers, int64_t K,
                            float* out, int64_t out_stride, int64_t out_offset, void* stream);
/* Its backward: for every valid slot, grad_src[b, idx, w] += g and (when
 * grad_centers is non-null) grad_centers[(b R + r) / K, w] -= g, g read from
 * grad_out with the same stride and offset.  Accumulates: the caller zeroes
 * grad_src and grad_centers. */
MPO_API int mpo_gather_rows_backward(const float* grad_out, int64_t out_stride,
                                     int64_t out_offset, int64_t B, int64_t N, int64_t W,
                                     const void* idx, int idx_int32, int64_t R, int64_t K,
                                     float* grad_src, float* grad_centers, void* stream);

/* Pointcept inverse-distance interpolation (mps_pointops/pointcept.py:219-243):
 * feat (N, C), the k nearest idx (M, k) int32 (-1 = none) and their distances
 * dist (M, k) from knn_query -> out (M, C):
 *   r_t = 1 / (dist_t + 1e-8) for valid t, else 0;  w_t = r_t / max(sum_t r_t, 1e-20);
 *   out[m, c] = sum_t w_t * feat[idx_t, c], each operation rounded, t in order.
 * Backward: grad_feat (N, C, overwritten) receives w_t * grad_out[m, c] at
 * idx_t (the weights carry no gradient, as in the reference). */
MPO_API int mpo_flat_interpolate(const float* feat, int64_t N, int64_t C, const int32_t* idx,
                                 const float* dist, int64_t M, int64_t k, float* out,
                                 void* stream);
MPO_API int mpo_flat_interpolate_backward(const float* grad_out, const int32_t* idx,
                                          const float* dist, int64_t M, int64_t k, int64_t N,
                                          int64_t C, float* grad_feat, void* stream);

/* ------------------------------------------------------------------ ranks
 * All-reduce (sum) of one float per rank over peer memory, for the loss of a
 * batch of Chamfer clouds split across the GPUs of one node (the reference is
 * single-device; this replaces the 4-byte NCCL all_reduce that would follow
 * its chamfer_distance, mps_pointops/chamfer.py:342-488, in a data-parallel
 * step).  Each rank creates one exchange array (mpo_p2p_slots_bytes() bytes
 * of device memory, zeroed) with mpo_p2p_slots_create, which also returns
 * its CUDA IPC handle (MPO_P2P_IPC_HANDLE_BYTES bytes); the ranks exchange the
 * handles (e.g. torch.distributed.all_gather_object) and map every other
 * rank's array with mpo_p2p_slots_open.
 *
 * mpo_allreduce_sum_f32_p2p: slots[r] = rank r's array as mapped in this
 * process (slots[rank] = the array this rank created), 1 <= world <=
 * MPO_P2P_MAX_RANKS.  Every rank makes the same sequence of calls with the
 * same seq (a counter that starts at 1, advances by one per call and skips
 * 0 when it wraps); each stores fl(value[0] * scale) into every rank's array
 * and waits until all W values have arrived in its own; out[0] = the W
 * values summed in rank order, each addition rounded -- the same bits on
 * every rank.  The wait is bounded: after timeout_ns without some rank's
 * value, out[0] = NaN and *status = 1 + the lowest missing rank (the caller
 * zeroes *status once; it is never cleared by the kernel).  One 32-thread
 * launch; calls on different ranks wait on one another, so each rank's call
 * must run on its own GPU.
 *
 * Teardown: once no call is in flight on any rank (synchronize, then a
 * barrier), close the mappings (mpo_p2p_slots_close), barrier again, then
 * free the own array (mpo_p2p_slots_destroy). */
#define MPO_P2P_MAX_RANKS 32
#define MPO_P2P_IPC_HANDLE_BYTES 64
MPO_API size_t mpo_p2p_slots_bytes(void);
MPO_API int mpo_p2p_slots_create(void** slots, void* ipc_handle);
MPO_API int mpo_p2p_slots_open(const void* ipc_handle, void** peer_slots);
MPO_API int mpo_p2p_slots_close(void* peer_slots);
MPO_API int mpo_p2p_slots_destroy(void* slots);
MPO_API int mpo_allreduce_sum_f32_p2p(const float* value, float scale, float* out,
                                      void* const* slots, int64_t world, int64_t rank,
                                      uint32_t seq, int64_t timeout_ns, int32_t* status,
                                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MPO_B200_H_ */
