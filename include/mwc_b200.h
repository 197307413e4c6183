/*
 * mwc_b200.h -- C ABI of the B200 (sm_100a) selective-scan library libmwc_b200.so.
 *
 * Drop-in native boundary for the hot path of zouyuanqing/mamba-windows-cuda
 * (N = 16 selective scan, forward + backward with h_prev / h_last streaming, and the
 * first-order linear-recurrence scan behind parallel_scan_fn). Every entry point takes
 * plain device pointers, int64 sizes, a dtype code and a cudaStream_t passed as void*.
 * Nothing is allocated inside the library: outputs and workspaces come from the caller
 * (the Python layer allocates them with the PyTorch caching allocator). Calls are
 * reentrant. Process-wide state: the per-thread error message and last-launch error word,
 * per-device caches (SM count, the kernels' shared-memory attribute), and the file-scope
 * device array of mwc_ss_fwd_noalloc (the only state shared between calls on the GPU).
 *
 * All tensors are contiguous row-major with these shapes (N = 16 states):
 *   u, delta, out, du, ddelta, dout : (B, L, D)
 *   A, dA : (D, 16)      Bm, Cm, dB, dC : (B, L, 16)      Dv, dD : (D)
 *   h_prev, h_last, dh_last, dh_prev : (B, D, 16)          (same dtype as u)
 *   ckpt  : (B, nck, D, 16) float32, nck = mwc_ss_ckpt_count(L); ckpt[b, k] is the state
 *           after step min(16 (k + 1), L) - 1
 *   decay, h_in : (B, D, 16) float32
 * All floating tensors of one call share one dtype (MWC_F32, MWC_F16 or MWC_BF16) except
 * the float32 ckpt / decay / h_in buffers; arithmetic is float32 throughout. (The
 * reference takes float32 / float16; bfloat16 I/O is an addition of this library.)
 *
 * Return value: MWC_OK (0) or an MWC_ERR_* code; mwc_last_error() then gives the message
 * (same wording as the reference's TORCH_CHECKs where one exists).
 */
#ifndef MWC_B200_H
#define MWC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MWC_ABI_VERSION 1

#if defined(__GNUC__)
#define MWC_API __attribute__((visibility("default")))
#else
#define MWC_API
#endif

enum mwc_dtype { MWC_F32 = 0, MWC_F16 = 1, MWC_BF16 = 2 };

enum mwc_status {
    MWC_OK = 0,
    MWC_ERR_INVALID = 1,    /* bad pointer, shape or dtype (reference: TORCH_CHECK -> RuntimeError) */
    MWC_ERR_UNSUPPORTED = 2,/* valid request this build does not implement */
    MWC_ERR_WORKSPACE = 3,  /* workspace missing or smaller than the *_workspace_bytes query */
    MWC_ERR_CUDA = 4,       /* a CUDA launch or runtime call failed */
    MWC_ERR_TIMEOUT = 5     /* a bounded device-side wait gave up (no GPU fault is raised) */
};

/* Library identity and error reporting. */
MWC_API int mwc_abi_version(void);
MWC_API const char* mwc_last_error(void);            /* message of the last failed call on this thread */
MWC_API const char* mwc_build_info(void);            /* compiler / arch string of this build */

/* Number of float32 checkpoint states per channel for a sequence of length L (ceil(L/16)). */
MWC_API int64_t mwc_ss_ckpt_count(int64_t L);

/* Workspace bytes mwc_ss_fwd needs for (B, L, D) on the current device: segment carries
 * when the sequence is split along L, or the work-queue flags and segment hand-off states
 * of the persistent kernel when B*D/128 reaches the SM count; 0 for a single pass. */
MWC_API int64_t mwc_ss_fwd_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype);

/*
 * Forward selective scan: h_t = exp(delta_t * A) h_{t-1} + delta_t u_t B_t,
 * out_t = <C_t, h_t> + Dv * u_t, h_{-1} = h_prev (or 0 when NULL).
 * Replaces selective_scan_cuda_forward / _forward_with_state / _forward_store
 * (mamba_windows_cuda/mamba_cuda.py:176-269, 271-359, 747-764) and
 * fused_selective_scan_forward (mamba_windows_cuda/selective_scan_cuda_ext.py:389-452).
 * Optional outputs (NULL to skip): out, h_last (dtype), ckpt (float32 states every 16 steps,
 * what the backward reads), decay = exp(A * sum_t delta_t) (float32, the segment decay an
 * L-sharded caller combines). out may be NULL to only produce checkpoints (recompute for
 * checkpoint level 1). The exponent is clamped to [-88, 88] like safe_exp
 * (mamba_cuda.py:65-70).
 */
MWC_API int mwc_ss_fwd(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
               const void* Dv, const void* h_prev, void* out, void* h_last, float* ckpt,
               float* decay, void* workspace, int64_t workspace_bytes,
               int64_t B, int64_t L, int64_t D, int dtype, void* stream);

/* Workspace bytes mwc_ss_bwd needs for (B, L, D) on the current device. */
MWC_API int64_t mwc_ss_bwd_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype);

/*
 * mwc_ss_plan -- the launch plan mwc_ss_fwd (backward = 0) or mwc_ss_bwd (backward = 1) picks
 * for (B, L, D, dtype) on the current device, assuming 16-byte-aligned buffers. Writes
 * info[0] = path (MWC_PATH_*), info[1] = K (time segments per 128-channel chain),
 * info[2] = segment length in time tiles (32 steps forward, 16 backward; the segmented
 * generic path: steps), info[3] = CTAs of the main launch. The chained forward
 * (MWC_PATH_CHAINED, backward = 0) instead gives each CTA one run of the chains'
 * concatenated tiles: info[2] is the longest run, and info[1] is 2 when a run boundary
 * cuts a chain (its head and tail run on two CTAs), else 1. For tests and tuning; no
 * counterpart in the reference (its kernels had one fixed launch shape).
 */
enum mwc_path { MWC_PATH_GENERIC = 0, MWC_PATH_CHAINED = 1, MWC_PATH_SPLIT = 2 };
MWC_API int mwc_ss_plan(int64_t B, int64_t L, int64_t D, int dtype, int backward, int32_t* info);

/*
 * Backward of mwc_ss_fwd for loss = sum(out * dout) + sum(h_last * dh_last): a reverse scan
 * that recomputes states chunk by chunk from ckpt (required when L > 16) and h_prev.
 * Produces du, ddelta (B, L, D), dA (D, 16), dB, dC (B, L, 16), dD (D) in dtype and, when
 * dh_prev != NULL, dh_prev (B, D, 16). dh_last may be NULL (zero). All reductions run in a
 * fixed order, so results are bitwise reproducible.
 * Replaces selective_scan_cuda_backward / _backward_direct (mamba_cuda.py:564-604, 766-790),
 * the stateful PyTorch backward selective_scan_backward (mamba_cuda.py:949-1041) and the
 * extension's selective_scan_backward (selective_scan_cuda_ext.py:454-514).
 */
MWC_API int mwc_ss_bwd(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
               const void* Dv, const void* h_prev, const void* dout, const void* dh_last,
               const float* ckpt, void* du, void* ddelta, void* dA, void* dB, void* dC, void* dD,
               void* dh_prev, void* workspace, int64_t workspace_bytes,
               int64_t B, int64_t L, int64_t D, int dtype, void* stream);

/*
 * Fold a known incoming state into a scan that was run from zero (sequence sharding along
 * L): with Pcum_t = exp(A * sum_{s<=t} delta_s),
 *   out_t  += <C_t, Pcum_t * h_in>            (out may be NULL)
 *   ckpt_k += Pcum_{t_k} * h_in               (ckpt may be NULL)
 *   h_last  = decay * h_in + h_last           (h_last may be NULL; decay required then)
 * The out/ckpt loop stops once every state has decayed below 2^-40 of h_in (never when an
 * exponent A*delta is positive or a delta is negative). No reference counterpart: the
 * reference has no sequence sharding; this is the carry fixup of the L-sharded scan.
 */
MWC_API int mwc_ss_fixup(const void* delta, const void* A, const void* Cm, const float* h_in,
                 const float* decay, void* out, void* h_last, float* ckpt,
                 int64_t B, int64_t L, int64_t D, int dtype, void* stream);

/*
 * Sequence sharding along L (no counterpart in the reference, which runs on one GPU): a rank
 * scans its time range from a zero state with mwc_ss_fwd_seq, which is mwc_ss_fwd plus
 * dprefix, float32 (B, mwc_ss_dprefix_count(L), D, 2): per 32-step tile and channel, the
 * delta prefix sum before the tile and the minimum over the tile's steps of the prefix sum
 * through each step (decay must be requested too). It is produced on the persistent path
 * (see mwc_ss_plan); other shapes return MWC_ERR_UNSUPPORTED, and the caller uses
 * mwc_ss_fixup. mwc_ss_fixup_chunked then applies the incoming state h_in like mwc_ss_fixup,
 * cut into 256-step chunks that run in parallel, each started from its prefix and skipped
 * exactly when the incoming state stays below 2^-40 throughout it.
 */
MWC_API int64_t mwc_ss_dprefix_count(int64_t L);
MWC_API int mwc_ss_fwd_seq(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
               const void* Dv, const void* h_prev, void* out, void* h_last, float* ckpt, float* decay,
               float* dprefix, void* workspace, int64_t workspace_bytes,
               int64_t B, int64_t L, int64_t D, int dtype, void* stream);
MWC_API int mwc_ss_fixup_chunked(const void* delta, const void* A, const void* Cm, const float* h_in,
               const float* decay, const float* dprefix, void* out, void* h_last, float* ckpt,
               int64_t B, int64_t L, int64_t D, int dtype, void* stream);

/*
 * mwc_ss_adjoint_seq -- the adjoint state at the start of a time range, float32 (B, D, 16):
 * q_L = q_in (NULL: zero), q_t = a_t (dout_t C_t + q_{t+1}), q_out = q_0, with
 * a_t = exp(min(delta_t A, 88)) per state: what a rank of a sequence-sharded backward hands
 * to the ranks before it, without the gradients of a full reverse scan (one exp and two
 * multiply-adds per element and state). Workspace: mwc_ss_adjoint_seq_workspace_bytes(B, L,
 * D) bytes, 16-byte aligned. No counterpart in the reference (single GPU).
 */
MWC_API int64_t mwc_ss_adjoint_seq_workspace_bytes(int64_t B, int64_t L, int64_t D);
MWC_API int mwc_ss_adjoint_seq(const void* delta, const void* A, const void* Cm, const void* dout,
               const float* q_in, float* q_out, void* workspace, int64_t workspace_bytes,
               int64_t B, int64_t L, int64_t D, int dtype, void* stream);

/*
 * mwc_ss_bwd_seq -- mwc_ss_bwd for one rank's range of a sequence-sharded scan, with the
 * states that cross range boundaries in float32 (B, D, 16): h_in, the state entering the
 * range (NULL: zero); q_in, the adjoint entering at the range end (NULL: zero); q_out, the
 * adjoint at the range start (NULL: not written). ckpt holds the range's true states (the
 * local scan's checkpoints after mwc_ss_fixup[_chunked] folded h_in into them). The rest is
 * mwc_ss_bwd's contract. No counterpart in the reference (single GPU).
 */
MWC_API int mwc_ss_bwd_seq(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
               const void* Dv, const float* h_in, const void* dout, const float* q_in,
               const float* ckpt, void* du, void* ddelta, void* dA, void* dB, void* dC, void* dD,
               float* q_out, void* workspace, int64_t workspace_bytes,
               int64_t B, int64_t L, int64_t D, int dtype, void* stream);

/*
 * mwc_ss_fwd_grouped / mwc_ss_bwd_grouped -- mwc_ss_fwd / mwc_ss_bwd with B_ssm and C_ssm (and
 * dB, dC) of shape (B, L, G, 16): channel d reads group d / (D / G). No counterpart in the
 * reference, whose B / C are (B, L, 16) (G = 1, where these equal mwc_ss_fwd / mwc_ss_bwd);
 * the official Mamba scan takes grouped B / C. G must divide D, D / G must be a multiple of
 * 128, and the shape must take the persistent path (16-byte-aligned buffers, rows of
 * D x element size a multiple of 16 bytes, and B*D/128 >= SM count or L >= 512); otherwise
 * MWC_ERR_UNSUPPORTED. Workspace sizes as for mwc_ss_fwd / mwc_ss_bwd.
 */
MWC_API int mwc_ss_fwd_grouped(const void* u, const void* delta, const void* A, const void* Bm,
               const void* Cm, const void* Dv, const void* h_prev, void* out, void* h_last,
               float* ckpt, float* decay, void* workspace, int64_t workspace_bytes,
               int64_t B, int64_t L, int64_t D, int64_t G, int dtype, void* stream);
MWC_API int mwc_ss_bwd_grouped(const void* u, const void* delta, const void* A, const void* Bm,
               const void* Cm, const void* Dv, const void* h_prev, const void* dout,
               const void* dh_last, const float* ckpt, void* du, void* ddelta, void* dA, void* dB,
               void* dC, void* dD, void* dh_prev, void* workspace, int64_t workspace_bytes,
               int64_t B, int64_t L, int64_t D, int64_t G, int dtype, void* stream);

/*
 * mwc_ss_fwd_nstate -- the forward scan of mwc_ss_fwd with N = 16, 32 or 64 states per channel:
 * A (D, N), B_ssm / C_ssm (B, L, N), h_prev / h_last / decay (B, D, N), ckpt (B, nck, D, N).
 * No counterpart in the reference, which supports N = 16 only (mamba_cuda.py:186-238 rejects
 * others); the official Mamba scan takes larger N. N = 16 is mwc_ss_fwd; N = 32 / 64 run the
 * generic forward kernels, forward only (there is no backward for them here). Workspace:
 * mwc_ss_fwd_nstate_workspace_bytes.
 */
MWC_API int64_t mwc_ss_fwd_nstate_workspace_bytes(int64_t B, int64_t L, int64_t D, int64_t N, int dtype);
MWC_API int mwc_ss_fwd_nstate(const void* u, const void* delta, const void* A, const void* Bm,
               const void* Cm, const void* Dv, const void* h_prev, void* out, void* h_last,
               float* ckpt, float* decay, void* workspace, int64_t workspace_bytes,
               int64_t B, int64_t L, int64_t D, int64_t N, int dtype, void* stream);

/*
 * First-order linear recurrence along axis 2 of (B, D, L, N) = (R, L, N) with R = B*D:
 * h_0 = x_0 (a_0 ignored), h_t = a_t h_{t-1} + x_t. Replaces PScan.forward /
 * parallel_scan_fn (mamba_windows_cuda/pscan.py:16-150), with the semantics of
 * parallel_scan_ref (pscan.py:153-171).
 */
MWC_API int mwc_lin_scan_fwd(const void* a, const void* x, void* h, int64_t R, int64_t L, int64_t N,
                     int dtype, void* stream);

/* Gradient of mwc_lin_scan_fwd for loss = sum(h * g): gx_t = g_t + a_{t+1} gx_{t+1},
 * ga_t = gx_t h_{t-1}, ga_0 = 0. Replaces PScan.backward (pscan.py:98-136). */
MWC_API int mwc_lin_scan_bwd(const void* a, const void* h, const void* g, void* ga, void* gx,
                     int64_t R, int64_t L, int64_t N, int dtype, void* stream);

/*
 * mwc_ss_fwd_noalloc -- the forward scan of mwc_ss_fwd (same arguments, same results) for
 * callers that cannot allocate device memory, such as foreign-language bindings that only
 * own their input and output buffers, or latency-bound loops where cudaMalloc's implicit
 * synchronization is not acceptable. It takes no workspace: the L-segment carries live in a
 * file-scope device array of 4 MiB that every GPU loading the library keeps until exit; a
 * shape that would need more is rejected with MWC_ERR_UNSUPPORTED. The first call on a device
 * looks up the array's address (make it before any stream capture). All calls on a device
 * share the array; each call rewrites what it reads, but calls that overlap on the GPU race.
 * Always runs the segmented forward kernels (never the persistent TMA kernel, whose
 * workspace grows with B*D). No counterpart in the reference: its ops always allocated
 * their outputs and scratch through the PyTorch allocator.
 */
MWC_API int mwc_ss_fwd_noalloc(const void* u, const void* delta, const void* A, const void* Bm,
                               const void* Cm, const void* Dv, const void* h_prev, void* out,
                               void* h_last, float* ckpt, float* decay,
                               int64_t B, int64_t L, int64_t D, int dtype, void* stream);

/*
 * Extended scan with the input / output transforms of Mamba's block (not in the reference,
 * which takes delta and returns y as they are; the official Mamba scan has these arguments):
 *   delta_eff = softplus(delta + delta_bias)   if delta_softplus, else delta + delta_bias
 *               (delta_bias: (D), NULL = 0; softplus(x) = log(1 + e^x), x for x > 20)
 *   out       = the selective scan of (u, delta_eff, A, Bm, Cm, Dv, h_prev)   (ungated y)
 *   out_z     = out * silu(z) = out * z / (1 + e^-z)          when z (B, L, D) is given
 * The backward takes dout with respect to out_z when z is given (else to out), the ungated
 * `out` of the forward (required with z) and returns dz and ddelta_bias (D) (both may be
 * NULL when not wanted). Layouts, dtypes and the other arguments as mwc_ss_fwd / _bwd;
 * ckpt is the forward's checkpoint buffer. Workspaces: the _workspace_bytes queries.
 */
MWC_API int64_t mwc_ss_fwd_ex_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype);
MWC_API int mwc_ss_fwd_ex(const void* u, const void* delta, const void* A, const void* Bm,
                          const void* Cm, const void* Dv, const void* z, const void* delta_bias,
                          int delta_softplus, const void* h_prev, void* out, void* out_z,
                          void* h_last, float* ckpt, void* workspace, int64_t workspace_bytes,
                          int64_t B, int64_t L, int64_t D, int dtype, void* stream);
MWC_API int64_t mwc_ss_bwd_ex_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype);
MWC_API int mwc_ss_bwd_ex(const void* u, const void* delta, const void* A, const void* Bm,
                          const void* Cm, const void* Dv, const void* z, const void* delta_bias,
                          int delta_softplus, const void* h_prev, const void* out,
                          const void* dout, const void* dh_last, const float* ckpt, void* du,
                          void* ddelta, void* dA, void* dB, void* dC, void* dD,
                          void* ddelta_bias, void* dz, void* dh_prev, void* workspace,
                          int64_t workspace_bytes, int64_t B, int64_t L, int64_t D, int dtype,
                          void* stream);

/*
 * Causal depthwise conv1d, the producer of u in Mamba's block (not in the reference; the
 * official Mamba stack ships it as causal_conv1d). Channel-last like the scan:
 *   x, y, dy, dx (B, L, D); weight, dweight (D, W), 1 <= W <= 4; bias, dbias (D) or NULL;
 *   x_prev, dx_prev (B, W-1, D) or NULL: the W-1 inputs before t = 0 (zero when NULL), for
 *   chunked streaming; activation 0 = none, 1 = SiLU.
 *   y[b,t,d] = act(bias[d] + sum_k weight[d,k] x[b, t-(W-1)+k, d])
 * The backward recomputes the pre-activation from x; dweight / dbias are reduced in a fixed
 * order (workspace: mwc_conv1d_bwd_workspace_bytes).
 */
MWC_API int mwc_conv1d_fwd(const void* x, const void* weight, const void* bias, const void* x_prev,
                           int activation, void* y, int64_t B, int64_t L, int64_t D, int64_t W,
                           int dtype, void* stream);
MWC_API int64_t mwc_conv1d_bwd_workspace_bytes(int64_t B, int64_t L, int64_t D, int64_t W);
MWC_API int mwc_conv1d_bwd(const void* x, const void* weight, const void* bias, const void* x_prev,
                           int activation, const void* dy, void* dx, void* dweight, void* dbias,
                           void* dx_prev, void* workspace, int64_t workspace_bytes, int64_t B,
                           int64_t L, int64_t D, int64_t W, int dtype, void* stream);

/*
 * mwc_check_last_launch -- waits for `stream` and reports whether the last persistent
 * forward / backward kernel launched from this thread gave up on a bounded device wait
 * (returns MWC_ERR_TIMEOUT, results of that call are invalid) or not (MWC_OK). The
 * workspace passed to that call must still be allocated. Calls that ran the segmented
 * kernels (which have no device waits) leave nothing to check: MWC_OK without touching
 * the device. No counterpart in the reference (its kernels had no device-side waits).
 */
MWC_API int mwc_check_last_launch(void* stream);

/*
 * mwc_selftest_wait_timeout -- launches one CTA whose bounded mbarrier wait can never be
 * satisfied (nothing arrives), with a short iteration limit, and reports what the host
 * reads back: MWC_ERR_TIMEOUT is the expected outcome (the wait expired, the kernel
 * recorded it in *dev_word and returned; the context stays usable), MWC_OK would mean the
 * wait did not expire. `dev_word`: 4 bytes of device memory owned by the caller. For the
 * failure-detection tests; no counterpart in the reference.
 */
MWC_API int mwc_selftest_wait_timeout(int* dev_word, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MWC_B200_H */
