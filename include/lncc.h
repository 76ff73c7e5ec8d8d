/*
 * lncc.h - C ABI of the B200 (sm_100a) fused 3-D LNCC loss library (liblncc_sm100.so).
 *
 * Every entry point is a plain C function: raw device pointers, sizes, a CUDA stream, and an int
 * status code (LNCC_OK == 0). No C++ exception crosses this boundary and no call allocates device
 * memory: the caller owns every buffer, including the scratch "workspace" whose size
 * lncc_workspace_bytes() reports. Work runs on the current device and is ordered on the caller's
 * stream: everything queued on that stream after a call sees all of its results. One exception to
 * "only on the caller's stream": for large calls lncc_fused_forward adds a second ("companion")
 * launch that runs concurrently on a stream the library makes for the calling host thread (with two
 * events) on its first such call, forked from and joined back into the caller's stream. To keep every
 * launch on the caller's stream, call lncc_set_companion(0) or use lncc_fused_forward_noalloc.
 *
 * Layout: pred/target/grad are contiguous (B, D, H, W) volumes, B = N*C, W fastest, fp32, bf16 or
 * fp16 (every type is loaded into fp32 registers; all arithmetic is fp32, the loss sum fp64).
 *
 * Math (reference fused_lncc/csrc/lncc3d.cu:5-8,93-108): for each voxel the k^3 zero-padded box
 * (n = k^3 at borders too) gives Sp, St, Spp, Stt, Spt;
 *   cross = Spt - Sp*St/n, var_p = max(Spp - Sp^2/n, 0) + dr, var_t = max(Stt - St^2/n, 0) + dr,
 *   cc = cross^2 / (var_p*var_t), clamped to 1 (NaN propagates), loss = 1 - mean(cc).
 * dL/dpred = -(1/M) * (box(A) + 2*pred*box(B) + target*box(C)) with the adjoints of
 * lncc3d.cu:100-107 (all zero where cc >= 1).
 */
#ifndef LNCC_SM100_H
#define LNCC_SM100_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. Mirrors the reference's TORCH_CHECK failure classes (lncc3d.cu:123,128-129,158,159). */
enum lncc_status {
  LNCC_OK = 0,
  LNCC_ERR_BAD_ARG = 1,         /* null pointer, non-positive size, bad plane range */
  LNCC_ERR_KERNEL_SIZE = 2,     /* kernel_size not in {3,5,7,9}  (lncc3d.cu:123) */
  LNCC_ERR_DTYPE = 3,           /* dtype not fp32/bf16/fp16      (lncc3d.cu:158) */
  LNCC_ERR_LAUNCH = 4,          /* kernel launch failed          (lncc3d.cu:159) */
  LNCC_ERR_SMEM = 5,            /* shared memory need above the device opt-in cap (lncc3d.cu:143-148) */
  LNCC_ERR_WORKSPACE = 6,       /* workspace missing or smaller than lncc_workspace_bytes() */
  LNCC_ERR_CUDA = 7,            /* other CUDA runtime error */
  LNCC_ERR_TOO_LARGE = 8,       /* size beyond a stated fixed maximum */
  LNCC_ERR_ABORTED = 9,         /* a bounded wait in the kernel timed out (lncc_check_abort) */
  LNCC_ERR_CHECK = 10           /* checked build only: a kernel index left its array */
};

/* Element types of pred / target / grad. The reference dispatches on fp32 and bf16 (lncc3d.cu:151-158)
 * and lists fp16 as open (BENCHMARKS.md:177-178); fp16 is handled exactly like bf16: loaded into
 * fp32, the gradient rounded to fp16 on store. */
enum lncc_dtype { LNCC_F32 = 0, LNCC_BF16 = 1, LNCC_F16 = 2 };

/* Human-readable text for a status code (static storage, never NULL). */
const char* lncc_strerror(int status);

/* Library version as major*10000 + minor*100 + patch. */
int lncc_version(void);

/*
 * Bytes of scratch the fused kernel needs for a call with these sizes: a 16-byte header (the abort
 * word read by lncc_check_abort) and one fp64 partial sum of cc per thread block. The reference allocates its four fp32 maps itself (lncc3d.cu:130-132); here the
 * only scratch is this small partials array (a few KB to a few hundred KB).
 * z_begin/z_end: output plane range (see lncc_fused_forward); pass 0, D for whole volumes.
 */
size_t lncc_workspace_bytes(int64_t B, int64_t D, int64_t H, int64_t W, int kernel_size, int dtype,
                            int64_t z_begin, int64_t z_end);

/*
 * One fused pass: reads pred and target once, writes the per-block cc partial sums, and (when
 * grad != NULL) writes dL/dpred in pred's dtype. Replaces the reference's lncc_forward
 * (lncc3d.cu:127-161) plus lncc_backward (lncc3d.cu:253-284) plus the torch `ncc.mean()` and
 * `* (-grad_out/M)` steps of fused_lncc/__init__.py:56-73: nothing is materialised in between.
 *
 *   pred, target : (B, D, H, W) device arrays of `dtype`.
 *   z_begin,z_end: only output planes [z_begin, z_end) of every volume are produced (loss terms and
 *                  grad). Planes outside the array are zero padding; planes inside it but outside
 *                  the range are read as halo. Whole volumes: 0, D. D-slab shards pass a slab with
 *                  2*(k/2) halo planes on each interior side.
 *   grad         : NULL (loss only, 8 B/voxel of traffic for fp32) or a (B, z_end-z_begin, H, W)
 *                  array of `dtype` that receives grad_scale * (*grad_scale_dev, if not NULL) *
 *                  d(sum cc)/dpred. For the loss 1 - mean(cc) pass grad_scale = -1/M.
 *   cc_sum_out   : NULL or one device double receiving sum(cc) over the produced voxels.
 *   loss_out     : NULL or one device float receiving 1 - sum(cc)/loss_count.
 *   workspace    : device scratch of at least lncc_workspace_bytes(...) bytes (8-byte aligned).
 * The cc sum is reduced in a fixed order: for the same launch plan (the same sizes, the same pointer
 * alignment, and the companion launch either taken or not) results are bitwise reproducible run to
 * run. Whether the companion runs (lncc_set_companion; inside a stream capture it runs only for a
 * thread that has made an eager companion-sized call before) changes the last bits of the volumes
 * it computes.
 */
int lncc_fused_forward(const void* pred, const void* target, int dtype,
                       int64_t B, int64_t D, int64_t H, int64_t W,
                       int kernel_size, float smooth_dr,
                       int64_t z_begin, int64_t z_end,
                       void* grad, float grad_scale, const float* grad_scale_dev,
                       double* cc_sum_out, float* loss_out, double loss_count,
                       void* workspace, size_t workspace_bytes, cudaStream_t stream);

/*
 * Status of the last lncc_fused_forward call that used `workspace`: LNCC_ERR_ABORTED when one of its
 * bounded waits (mbarrier waits of the warp-specialised kernel, 2 s each) ran out, in which case its
 * gradient and loss are invalid (the loss is also NaN), else LNCC_OK. The kernel leaves its loops
 * and returns after a timeout, so the CUDA context stays usable. Synchronises `stream` and reads
 * the workspace's first word; call it after that call, on the same stream. No counterpart in the
 * reference, whose kernels have no waits.
 */
int lncc_check_abort(const void* workspace, cudaStream_t stream);

/*
 * 1 when this library is the bounds-checked build (compiled with LNCC_CHECKED=1, `build.py --checked`,
 * file liblncc_sm100_checked.so), else 0. In the checked build every global, shared and tensor-memory
 * access of the kernels is range-checked; an access outside its array is skipped and counted, and
 * every entry point that launches kernels synchronises its stream and returns LNCC_ERR_CHECK when
 * the count is not zero. It stands in for compute-sanitizer runs (the reference's
 * tests/_sanitize2.py, tests/_sanitize_bf16.py). No counterpart in the reference.
 */
int lncc_checked_build(void);

/*
 * Self-test of the bounded wait: one warp waits on an mbarrier that nothing completes, gives up after
 * limit_us microseconds (1 .. 10^7) and records the abort in the workspace header exactly as the
 * fused kernel does, so that lncc_check_abort then returns LNCC_ERR_ABORTED. Diagnostics.
 */
int lncc_wait_timeout_selftest(void* workspace, size_t workspace_bytes, unsigned limit_us, cudaStream_t stream);

/*
 * Loss of a batch whose volumes are sharded over `world` ranks of one node, one GPU each, without a
 * collective library: a compute result followed by its reduction over NVLink peer memory in one
 * small kernel. Each rank calls it on its own stream after lncc_fused_forward wrote its shard's
 * sum of cc to local_sum (cc_sum_out). The kernel writes that sum into slot `rank` of every rank's
 * exchange buffer, waits (bounded, 2 s) until every rank's sum of this epoch has arrived in its own
 * buffer, and writes the same global sum (added in rank order, bitwise equal on every rank) and
 * loss = 1 - sum / count on every rank.
 *   slots : device array of `world` device pointers, slots[r] = rank r's exchange buffer mapped into
 *           this process (CUDA IPC), lncc_peer_exchange_bytes(world) bytes each, zeroed once.
 *   epoch : 1, 2, 3, ... one per call, the same on every rank.
 *   abort_word: NULL or a device word set to 1 when another rank's sum did not arrive in time (the
 *           sum and loss are then NaN).
 * Replaces the fp64 all-reduce of the cc sum (no counterpart in the reference, which has no
 * multi-GPU code).
 */
size_t lncc_peer_exchange_bytes(int world);
int lncc_peer_loss(const double* local_sum, void* const* slots, int rank, int world, uint64_t epoch,
                   double count, double* cc_sum_out, float* loss_out, unsigned* abort_word,
                   cudaStream_t stream);

/*
 * In place grad *= *grad_out for n elements of `dtype`; every block returns at once when
 * *grad_out == 1 (the usual loss.backward() case), so that case costs one tiny launch.
 * Replaces the `* (-grad_out / ctx.M)` tensor multiply of fused_lncc/__init__.py:73 (the -1/M part
 * is already folded into lncc_fused_forward's grad_scale).
 */
int lncc_scale_grad(void* grad, int dtype, int64_t n, const float* grad_out_dev, cudaStream_t stream);

/*
 * lncc_fused_forward without a caller-provided workspace. No counterpart in the reference. It is
 * for callers that cannot call cudaMalloc, for example code running where the allocator is owned by
 * someone else (a framework's caching allocator or a pool that must not grow), or where allocating
 * is forbidden at that point (inside a tight real-time loop). The scratch that lncc_fused_forward
 * takes as `workspace` here is a fixed array in the library's device memory: 65536 fp64 partial sums
 * (512 KiB) per GPU, held until the process exits. Sizes that need more than that return
 * LNCC_ERR_TOO_LARGE; lncc_workspace_bytes() tells how much a call needs. Nothing is allocated: the
 * first call on each device only looks up the array's device address (cudaGetSymbolAddress) with
 * that device current, so make that first call before capturing a stream into a CUDA graph. All
 * calls share the one array: calls that overlap on the GPU (different streams, no ordering) race.
 * It always runs as a single launch on `stream` (never the companion launch of lncc_set_companion,
 * which makes a stream and events of its own on first use).
 * Every other argument means exactly what it means for lncc_fused_forward.
 */
int lncc_fused_forward_noalloc(const void* pred, const void* target, int dtype,
                               int64_t B, int64_t D, int64_t H, int64_t W,
                               int kernel_size, float smooth_dr,
                               int64_t z_begin, int64_t z_end,
                               void* grad, float grad_scale, const float* grad_scale_dev,
                               double* cc_sum_out, float* loss_out, double loss_count,
                               cudaStream_t stream);

/*
 * Materialising compat path: the reference extension's three entry points with their outputs, for
 * debugging and for code written against them (the reference's own tests call them directly,
 * tests/test_pytest.py:38-51, tests/verify_fwd.py:20-24). The fused entry point above is the
 * training path; these write full fp32 maps (16 B/voxel for the forward).
 *
 * lncc_maps_forward replaces fused_lncc_cuda.lncc_forward (lncc3d.cu:127-161): from (B, D, H, W)
 * pred/target of `dtype` it writes four fp32 (B, D, H, W) maps: ncc (cc clamped to 1, NaN kept) and
 * the adjoints A = dncc/dSp, Bc = dncc/dvar_p, Cc = dncc/dcross of lncc3d.cu:100-107 (zero where
 * cc >= 1 or NaN). Any of ncc/A/Bc/Cc may be NULL to skip that map.
 */
int lncc_maps_forward(const void* pred, const void* target, int dtype,
                      int64_t B, int64_t D, int64_t H, int64_t W,
                      int kernel_size, float smooth_dr,
                      float* ncc, float* A, float* Bc, float* Cc, cudaStream_t stream);

/*
 * Replaces fused_lncc_cuda.lncc_backward (lncc3d.cu:253-284): writes
 * grad = scale * (box(A) + 2*pred*box(Bc) + target*box(Cc)) in `dtype` (pred's), for fp32 maps A, Bc,
 * Cc and pred/target of `dtype`, all (B, D, H, W).
 */
int lncc_maps_backward(const float* A, const float* Bc, const float* Cc,
                       const void* pred, const void* target, int dtype,
                       int64_t B, int64_t D, int64_t H, int64_t W,
                       int kernel_size, float scale, void* grad, cudaStream_t stream);

/*
 * Replaces fused_lncc_cuda.box3d_sep_forward (lncc3d.cu:329-344): y = zero-padded k^3 box sum of the
 * fp32 (B, D, H, W) array x. y must not overlap x.
 */
int lncc_box3d(const float* x, float* y, int64_t B, int64_t D, int64_t H, int64_t W, int kernel_size,
               cudaStream_t stream);

/*
 * Per-voxel loss (reduction 'none'), a feature the reference lists as open (BENCHMARKS.md:177-178)
 * and has no entry point for. lncc_loss_map_forward writes loss_map = 1 - ncc at every voxel, fp32
 * (B, D, H, W), with ncc clamped to 1 and NaN kept exactly as in lncc_maps_forward.
 * lncc_loss_map_backward writes grad = d(sum_v G(v) * loss_map(v))/dpred = -sum_v G(v) dncc(v)/dpred
 * in pred's dtype for an upstream fp32 (B, D, H, W) map G (grad_map): the adjoints of every voxel are
 * weighted by G there, then boxed as in lncc_maps_backward. It materialises three fp32 maps in the
 * caller's scratch of lncc_loss_map_scratch_bytes() bytes (12 bytes per voxel).
 */
size_t lncc_loss_map_scratch_bytes(int64_t B, int64_t D, int64_t H, int64_t W);
int lncc_loss_map_forward(const void* pred, const void* target, int dtype,
                          int64_t B, int64_t D, int64_t H, int64_t W,
                          int kernel_size, float smooth_dr, float* loss_map, cudaStream_t stream);
int lncc_loss_map_backward(const float* grad_map, const void* pred, const void* target, int dtype,
                           int64_t B, int64_t D, int64_t H, int64_t W,
                           int kernel_size, float smooth_dr, void* grad,
                           float* scratch, size_t scratch_bytes, cudaStream_t stream);

/*
 * Non-cubic windows kd x kh x kw (depth, height, width; each side odd, 1 .. 9; n = kd*kh*kw), a
 * feature the reference lists as open (BENCHMARKS.md:177-178) and has no entry point for. The window
 * replaces the k^3 cube everywhere in the math above (zero padding, n counted as the full window at
 * the borders, the same clamps), so a cubic (k, k, k) gives lncc_fused_forward's results.
 *
 * lncc_aniso_forward: every argument as for lncc_fused_forward (whole volumes: no plane range). One
 * pass writes the adjoint maps (three fp32 maps, only when grad != NULL) and one fp64 cc sum per
 * thread block into `scratch`; a fixed-order reduction gives cc_sum_out / loss_out; a second pass
 * boxes the maps into grad = grad_scale * (*grad_scale_dev if not NULL) * d(sum cc)/dpred. scratch:
 * lncc_aniso_scratch_bytes(B, D, H, W, grad != NULL) bytes, 8-byte aligned (12 bytes per voxel with
 * the gradient, a few KB without). This path materialises maps, unlike the fused kernel: about 60
 * bytes of traffic per voxel against 12.
 * lncc_aniso_loss_map_forward / _backward: lncc_loss_map_forward / _backward for such a window
 * (reduction 'none'; scratch of lncc_loss_map_scratch_bytes()).
 * A side outside 1 .. 9 or even returns LNCC_ERR_KERNEL_SIZE.
 */
size_t lncc_aniso_scratch_bytes(int64_t B, int64_t D, int64_t H, int64_t W, int with_grad);
int lncc_aniso_forward(const void* pred, const void* target, int dtype,
                       int64_t B, int64_t D, int64_t H, int64_t W,
                       int kd, int kh, int kw, float smooth_dr,
                       void* grad, float grad_scale, const float* grad_scale_dev,
                       double* cc_sum_out, float* loss_out, double loss_count,
                       void* scratch, size_t scratch_bytes, cudaStream_t stream);
int lncc_aniso_loss_map_forward(const void* pred, const void* target, int dtype,
                                int64_t B, int64_t D, int64_t H, int64_t W,
                                int kd, int kh, int kw, float smooth_dr, float* loss_map, cudaStream_t stream);
int lncc_aniso_loss_map_backward(const float* grad_map, const void* pred, const void* target, int dtype,
                                 int64_t B, int64_t D, int64_t H, int64_t W,
                                 int kd, int kh, int kw, float smooth_dr, void* grad,
                                 float* scratch, size_t scratch_bytes, cudaStream_t stream);

/*
 * Kernel selection for the whole process (diagnostics and cross-checks): 0 = automatic (default:
 * the warp-specialised cluster kernel when W % 4 == 0 and the pointers are aligned to 4 elements,
 * else the general sweep kernel), 1 = always the general sweep kernel, 3 = warp-specialised kernel
 * where supported. 2 named an earlier cluster kernel that has been retired; it returns
 * LNCC_ERR_BAD_ARG. No counterpart in the reference, which has a single kernel per step.
 */
int lncc_select_kernel(int which);

/*
 * Companion launch of the warp-specialised kernel (default on): clusters of 8 CTAs at one CTA per SM
 * do not tile every GPC of a B200 (15 clusters = 120 of 148 SMs), so when a call has enough volumes
 * the last few go to clusters of 2 CTAs on the idle SMs, run concurrently on a library-owned stream
 * that is forked from and joined back into the caller's stream. 0 turns it off for the process.
 * Returns the previous setting. No counterpart in the reference.
 */
int lncc_set_companion(int enable);

/*
 * Kernel launches lncc_fused_forward makes for this shape with 16-byte-aligned tensors, not counting
 * the loss reduction: 2 when the companion launch runs, else 1; or minus an LNCC_ERR_* status for bad
 * arguments. Diagnostics.
 */
int lncc_launch_count(int64_t B, int64_t D, int64_t H, int64_t W, int kernel_size, int dtype,
                      int64_t z_begin, int64_t z_end, int grad);

#ifdef __cplusplus
}
#endif

#endif /* LNCC_SM100_H */
