/*
 * mhc_b200.h -- C ABI of the B200 (sm_100a) mHC operator library.
 *
 * The reference (liuhycs/FlagOS-mhc) exposes these operators only as Python
 * functions on torch tensors; it has no FFI.  Each entry point below is the
 * device-side body of one of those Python functions, reduced to plain device
 * pointers, sizes and a CUDA stream, so any host language can bind it
 * (ctypes / cffi / cgo / JNI).  Tensor allocation stays with the caller.
 *
 * Conventions
 *   - All pointers are device pointers of contiguous row-major tensors.
 *     Tokens are flattened: a (B,S,N,D) tensor is passed as (T=B*S,N,D).
 *   - `dtype` names the element type of x / h_out / out / grad_y / grad_x /
 *     grad_h_out / y (MHC_F32, MHC_F16, MHC_BF16).  Every other tensor is fp32.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls are
 *     stream-ordered, never synchronise the host and are safe to call
 *     concurrently on different streams; the only process-wide state is a
 *     per-device attribute cache and the launch counter below.
 *   - Return value: 0 (MHC_OK) or an MHC_ERR_* code; mhc_status_string()
 *     turns it into text.  Argument checks run before any launch, so a
 *     non-zero return from a check leaves every output untouched.
 */
#ifndef MHC_B200_H_
#define MHC_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum mhc_dtype { MHC_F32 = 0, MHC_F16 = 1, MHC_BF16 = 2 };

enum mhc_status {
  MHC_OK = 0,
  MHC_ERR_INVALID_ARGUMENT = 1,  /* bad size, null pointer, bad scalar     */
  MHC_ERR_UNSUPPORTED_N = 2,     /* hcMult outside 1..8                     */
  MHC_ERR_UNSUPPORTED_DTYPE = 3, /* dtype not one of enum mhc_dtype         */
  MHC_ERR_WORKSPACE = 4,         /* workspace null / too small / misaligned */
  MHC_ERR_CUDA = 5,              /* a CUDA runtime call or launch failed    */
  MHC_ERR_DEVICE = 6,            /* current device is not sm_100            */
  MHC_ERR_TIMEOUT = 7,           /* a bounded device-side wait gave up      */
  MHC_ERR_SCRATCH_LIMIT = 8      /* needs more than the static scratch holds */
};

/* Text for a status code (static storage). */
const char* mhc_status_string(int status);

/* Library ABI version (major*10000 + minor*100 + patch). */
int mhc_version(void);

/* Running count of CUDA kernels this library has launched in this process
 * (all devices, all threads).  Diagnostic: lets a caller verify that the
 * device path ran.  No counterpart in the reference. */
uint64_t mhc_kernel_launches(void);

/* Synchronises the current device, then returns (and clears) the status a
 * tensor-core kernel recorded when one of its bounded device-side waits gave
 * up (MHC_ERR_TIMEOUT), MHC_ERR_CUDA if the device reports an error, else
 * MHC_OK.  Diagnostic; the operators themselves never synchronise.  No
 * counterpart in the reference. */
int mhc_device_status(void);

/* Self-test of the failure path: launches one CTA that waits on an mbarrier
 * phase nothing completes, with the bounded wait every tensor-core kernel of
 * this library uses, cut to `spin_limit` polls.  The wait gives up, the kernel
 * records MHC_ERR_TIMEOUT and returns; the next mhc_device_status() reports it
 * and the context stays usable.  Diagnostic; no counterpart in the reference. */
int mhc_selftest_wait_timeout(uint32_t spin_limit, void* stream);

/*
 * mhc_post forward.  Replaces the device work of `mhc_post`
 * (src/mhc_post.py:296-341, kernels :24-96 and :207-271):
 *   out[t,i,d] = sum_j h_res[t,j,i] * x[t,j,d] + h_post[t,i] * h_out[t,d]
 * x, out: (T,N,D) dtype.  h_res: (T,N,N) fp32.  h_out: (T,D) dtype.
 * h_post: (T,N) fp32.  Accumulation in fp32, one rounding on store.
 */
int mhc_post_fwd(const void* x, const float* h_res, const void* h_out,
                 const float* h_post, void* out, int64_t T, int32_t N,
                 int64_t D, int32_t dtype, void* stream);

/*
 * mhc_post backward.  Replaces `mhc_post_backward`
 * (src/mhc_post_backward.py:593-621, kernel :293-421):
 *   grad_x[t,j,d]    = sum_i h_res[t,j,i] * grad_y[t,i,d]     (dtype)
 *   grad_h_res[t,j,i]= sum_d x[t,j,d] * grad_y[t,i,d]         (fp32)
 *   grad_h_out[t,d]  = sum_i h_post[t,i] * grad_y[t,i,d]      (dtype)
 *   grad_h_post[t,i] = sum_d h_out[t,d] * grad_y[t,i,d]       (fp32)
 */
int mhc_post_bwd(const void* grad_y, const void* x, const float* h_res,
                 const void* h_out, const float* h_post, void* grad_x,
                 float* grad_h_res, void* grad_h_out, float* grad_h_post,
                 int64_t T, int32_t N, int64_t D, int32_t dtype,
                 void* stream);

/* Bytes of device workspace mhc_pre_fwd needs for these sizes. */
size_t mhc_pre_fwd_workspace_bytes(int64_t T, int32_t N, int64_t D,
                                   int32_t dtype);

/*
 * mhc_pre_clamp_sinkhorn forward.  Replaces `mhc_pre_clamp_sinkhorn`
 * (src/mhc_pre_clamp_sinkhorn.py:857-971; semantics :974-1022):
 *   inv = rsqrt(mean(x^2) + norm_eps) over N*D;  mixes = (x*inv) phi^T
 *   pre = sigmoid(mixes[:N]*a0 + b[:N]) + hc_eps
 *   post_out = 2*sigmoid(mixes[N:2N]*a1 + b[N:2N])
 *   logits = mixes[2N:]*a2 + b[2N:]  (N,N), clamped iff clamp_min!=0||clamp_max!=0
 *   comb = Sinkhorn(softmax_row(logits)), iter_times iterations
 *   y[t,d] = sum_n x[t,n,d] * pre[t,n]
 * x: (T,N,D) dtype; phi: (N*(N+2), N*D) fp32; alpha (3,); base (N*(N+2),).
 * Outputs: y (T,D) dtype; post_out (T,N); comb_frag (T,N,N); inv_rms (T,);
 * mixes (T,N*(N+2)); pre (T,N); optional (may be NULL): x_scaled (T,N*D),
 * h_res_logits (T,N,N, pre-clamp).  workspace: >= mhc_pre_fwd_workspace_bytes,
 * 256-byte aligned; its contents on entry do not matter.
 */
int mhc_pre_fwd(const void* x, const float* phi, const float* alpha,
                const float* base, int64_t T, int32_t N, int64_t D,
                int32_t dtype, float norm_eps, float hc_eps, float clamp_min,
                float clamp_max, int32_t iter_times, void* y, float* post_out,
                float* comb_frag, float* inv_rms, float* x_scaled,
                float* mixes, float* h_res_logits, float* pre, void* workspace,
                size_t workspace_bytes, void* stream);

/* Bytes of device workspace mhc_pre_bwd needs for these sizes. */
size_t mhc_pre_bwd_workspace_bytes(int64_t T, int32_t N, int64_t D,
                                   int32_t dtype, int32_t iter_times);

/*
 * mhc_pre_clamp_sinkhorn backward.  Replaces
 * `mhc_pre_clamp_sinkhorn_backward`
 * (src/mhc_pre_clamp_sinkhorn_backward.py:1292-1391; oracle :1397-1453).
 * Inputs are the tensors the forward saved (x, phi, alpha, base, inv_rms,
 * mixes, pre) and the upstream grads grad_y (T,D) dtype, grad_post_out (T,N),
 * grad_comb_frag (T,N,N).  x_scaled and h_res_logits are not needed: the
 * kernels recompute x*inv_rms on the fly and the logits from mixes.
 * Outputs: grad_x (T,N,D) dtype; grad_phi (N*(N+2), N*D); grad_alpha (3,);
 * grad_base (N*(N+2),).  All reductions run in a fixed order (no float
 * atomics), so the result is bitwise reproducible run to run.
 */
int mhc_pre_bwd(const void* x, const float* phi, const float* alpha,
                const float* base, const float* inv_rms, const float* mixes,
                const float* pre, const void* grad_y,
                const float* grad_post_out, const float* grad_comb_frag,
                int64_t T, int32_t N, int64_t D, int32_t dtype,
                float norm_eps, float hc_eps, float clamp_min, float clamp_max,
                int32_t iter_times, void* grad_x, float* grad_phi,
                float* grad_alpha, float* grad_base, void* workspace,
                size_t workspace_bytes, void* stream);

/*
 * mhc_pre_bwd_accumulate -- mhc_pre_bwd that adds an existing gradient into
 * grad_x: grad_x = (this operator's grad_x, fp32) + grad_x_accumulate, rounded
 * once to dtype.  No counterpart in the reference, whose callers let autograd
 * add the post and pre contributions to x's gradient in a separate pass (three
 * more x-sized transfers); src/autograd.py:14-87 is where that sum arises.
 * grad_x_accumulate has grad_x's shape and dtype and may be the same buffer
 * as grad_x (in-place accumulation).  Everything else is as mhc_pre_bwd.
 */
int mhc_pre_bwd_accumulate(const void* x, const float* phi, const float* alpha,
                           const float* base, const float* inv_rms,
                           const float* mixes, const float* pre,
                           const void* grad_y, const float* grad_post_out,
                           const float* grad_comb_frag, int64_t T, int32_t N,
                           int64_t D, int32_t dtype, float norm_eps,
                           float hc_eps, float clamp_min, float clamp_max,
                           int32_t iter_times, const void* grad_x_accumulate,
                           void* grad_x, float* grad_phi, float* grad_alpha,
                           float* grad_base, void* workspace,
                           size_t workspace_bytes, void* stream);

/*
 * Cross-GPU sum of the pre operator's parameter gradients over NVLink peer
 * memory (token-sharded data parallelism, one process per GPU).  No
 * counterpart in the reference, which has no distributed code: it replaces the
 * NCCL all-reduce of the packed [grad_phi | grad_alpha | grad_base] vector that
 * a data-parallel caller would run after mhc_pre_bwd (the sum of the per-rank
 * terms of the reference's grad_phi = torch.mm(grad_mixes.t(), x_scaled),
 * src/mhc_pre_clamp_sinkhorn_backward.py:1372-1373).
 *
 * Set-up, once per job (collective over the ranks, host side):
 *   each rank  mhc_peer_region_alloc(n, &region)       (cudaMalloc, zeroed)
 *              mhc_peer_handle(region, handle)           (CUDA IPC handle,
 *                                                        mhc_peer_handle_bytes())
 *   exchange the handles (any host channel), then for every other rank p
 *              mhc_peer_open(handle_p, &regions[p]);    regions[rank] = region
 * Per call (all ranks, same n, same order of calls):
 *   mhc_grad_sum_peers(src, dst, n, regions, rank, world, epoch, timeout_ns, s)
 * epoch: 0 = the kernel takes the call's epoch from a counter in this rank's region
 * (device memory; it advances once per call), so the call can be captured in a CUDA
 * graph and replayed; nonzero = the host numbers the calls 1, 2, 3, ... on every rank.
 * Use one of the two forms for the life of a set of regions.
 * writes the sum over the ranks of src (n floats) into dst (may equal src), in
 * rank order, so every rank gets bitwise the same vector.  One kernel launch,
 * stream-ordered.  Every wait for a peer gives up after timeout_ns; the kernel
 * then records MHC_ERR_TIMEOUT (returned by mhc_device_status), dst is not
 * valid, and the regions must be re-created before the next call.
 * Tear-down: mhc_peer_close on every opened peer region, a host barrier, then
 * mhc_peer_region_free.  world <= 8; src and dst 16-byte aligned.
 */
size_t mhc_peer_region_bytes(int64_t n);
int mhc_peer_region_alloc(int64_t n, void** region);
int mhc_peer_region_free(void* region);
int mhc_peer_handle_bytes(void);
int mhc_peer_handle(void* region, void* handle_out);
int mhc_peer_open(const void* handle, void** peer_region);
int mhc_peer_close(void* peer_region);
int mhc_grad_sum_peers(const float* src, float* dst, int64_t n,
                       void* const* regions, int32_t rank, int32_t world,
                       uint32_t epoch, uint64_t timeout_ns, void* stream);

/*
 * Token-strided forms of the four operators.  Same computation, arguments and
 * outputs as the entry points above, plus the number of ELEMENTS between the
 * first elements of consecutive tokens of the named inputs (x: >= N*D;
 * grad_y of mhc_post_bwd: >= N*D; h_out and the pre operator's grad_y: >= D).
 * Within a token the (N, D) block (or the D row) must be contiguous; outputs are
 * always packed.  This is how a (B,S,N,D) view whose B and S strides are
 * jointly regular (stride_B == S * stride_S), or a (T,N,D) slice of a larger
 * buffer, runs without a copy: the reference's backward passes x.stride(1) /
 * grad_y.stride(1) to its kernels the same way
 * (src/mhc_pre_clamp_sinkhorn_backward.py:1320-1344).  Tensor-core paths need
 * every token row 16-byte aligned (stride * element size a multiple of 16);
 * other strides run the general kernels.
 */
int mhc_post_fwd_strided(const void* x, int64_t x_token_stride, const float* h_res,
                         const void* h_out, int64_t h_out_token_stride,
                         const float* h_post, void* out, int64_t T, int32_t N,
                         int64_t D, int32_t dtype, void* stream);
int mhc_post_bwd_strided(const void* grad_y, int64_t grad_y_token_stride,
                         const void* x, int64_t x_token_stride,
                         const float* h_res, const void* h_out,
                         int64_t h_out_token_stride, const float* h_post,
                         void* grad_x, float* grad_h_res, void* grad_h_out,
                         float* grad_h_post, int64_t T, int32_t N, int64_t D,
                         int32_t dtype, void* stream);
int mhc_pre_fwd_strided(const void* x, int64_t x_token_stride, const float* phi,
                        const float* alpha, const float* base, int64_t T,
                        int32_t N, int64_t D, int32_t dtype, float norm_eps,
                        float hc_eps, float clamp_min, float clamp_max,
                        int32_t iter_times, void* y, float* post_out,
                        float* comb_frag, float* inv_rms, float* x_scaled,
                        float* mixes, float* h_res_logits, float* pre,
                        void* workspace, size_t workspace_bytes, void* stream);
/* grad_x_accumulate may be NULL (then this is mhc_pre_bwd with strides). */
int mhc_pre_bwd_strided(const void* x, int64_t x_token_stride, const float* phi,
                        const float* alpha, const float* base,
                        const float* inv_rms, const float* mixes,
                        const float* pre, const void* grad_y,
                        int64_t grad_y_token_stride, const float* grad_post_out,
                        const float* grad_comb_frag, int64_t T, int32_t N,
                        int64_t D, int32_t dtype, float norm_eps, float hc_eps,
                        float clamp_min, float clamp_max, int32_t iter_times,
                        const void* grad_x_accumulate, void* grad_x,
                        float* grad_phi, float* grad_alpha, float* grad_base,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Layer-level fusion of the forward pass (N = 4, bf16 / fp16, D % 64 == 0, packed
 * tensors).  No counterpart in the reference: in a stack of layers its callers
 * (src/autograd.py:14-87) run mhc_post for layer l, whose output x_{l+1} the
 * pre operator of layer l+1 then reads again for x.phi^T and sum(x^2)
 * (src/mhc_pre_clamp_sinkhorn.py:897-903).
 *
 * mhc_post_fwd_mix is mhc_post_fwd (out is bitwise the same) that also writes
 * `premix`, [layers][T][N*(N+2)+1] fp32: per K range (layers =
 * mhc_post_fwd_mix_layers) and token, the raw mix x_{l+1}.phi_next^T and the sum
 * of squares, computed from out while it is written.  mhc_pre_fwd_premixed is
 * mhc_pre_fwd of layer l+1 given those partials instead of phi: it reads x only
 * for y / x_scaled.  phi_next must be the phi that layer l+1 uses.
 * mhc_post_fwd_mix_supported says whether the fused path applies to a shape.
 */
int mhc_post_fwd_mix_supported(int64_t T, int32_t N, int64_t D, int32_t dtype);
int32_t mhc_post_fwd_mix_layers(int64_t T, int32_t N, int64_t D, int32_t dtype);
size_t mhc_post_fwd_mix_workspace_bytes(int64_t T, int32_t N, int64_t D,
                                        int32_t dtype);
int mhc_post_fwd_mix(const void* x, const float* h_res, const void* h_out,
                     const float* h_post, void* out, int64_t T, int32_t N,
                     int64_t D, int32_t dtype, const float* phi_next,
                     float* premix, void* workspace, size_t workspace_bytes,
                     void* stream);
int mhc_pre_fwd_premixed(const void* x, const float* premix,
                         int32_t premix_layers, const float* alpha,
                         const float* base, int64_t T, int32_t N, int64_t D,
                         int32_t dtype, float norm_eps, float hc_eps,
                         float clamp_min, float clamp_max, int32_t iter_times,
                         void* y, float* post_out, float* comb_frag,
                         float* inv_rms, float* x_scaled, float* mixes,
                         float* h_res_logits, float* pre, void* stream);

/* Size of the static device scratch array used by mhc_pre_fwd_noalloc. */
#define MHC_PRE_FWD_NOALLOC_SCRATCH_BYTES (16u << 20)

/*
 * mhc_pre_fwd_noalloc -- no counterpart in the reference.
 * Same computation, arguments and outputs as mhc_pre_fwd, but without the
 * workspace arguments: the scratch lives in a static 16 MiB device array of
 * this library, so the call allocates no device memory.  For callers that may
 * not call cudaMalloc where they run the operator (an arena or pooled
 * allocator that owns the device budget; a cgo/JNI/C binding with no device
 * allocator).  Returns MHC_ERR_SCRATCH_LIMIT when
 * mhc_pre_fwd_workspace_bytes(T,N,D,dtype) exceeds the array: N=4 at D <= 7168
 * fits up to T = 167,770 tokens (any dtype), N=8 at D = 4096 up to T = 51,780
 * (16-bit x; fp32 x: up to D = 2048), and N=8 at D = 7168 never fits.  All calls on a device share the array: calls that
 * overlap on the GPU race.  Every call made outside stream capture looks the
 * array's address up for the current device and context (so a context re-created
 * after cudaDeviceReset is handled); a call inside a capture reuses the address of
 * the last uncaptured call on the device, so make one call on each device before
 * any capture begins, and again after a cudaDeviceReset.
 */
int mhc_pre_fwd_noalloc(const void* x, const float* phi, const float* alpha,
                        const float* base, int64_t T, int32_t N, int64_t D,
                        int32_t dtype, float norm_eps, float hc_eps,
                        float clamp_min, float clamp_max, int32_t iter_times,
                        void* y, float* post_out, float* comb_frag,
                        float* inv_rms, float* x_scaled, float* mixes,
                        float* h_res_logits, float* pre, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MHC_B200_H_ */
