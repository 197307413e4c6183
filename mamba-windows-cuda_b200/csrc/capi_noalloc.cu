// mwc_ss_fwd_noalloc: the forward selective scan for callers that cannot allocate device
// memory. Some callers only own the buffers they pass in: foreign-language bindings that
// have no handle on a CUDA allocator, and latency-bound loops that must not call cudaMalloc
// (it can synchronize the device). This entry point takes the same inputs and outputs as
// mwc_ss_fwd but no workspace: the L-segment carries of the segmented forward scan
// (ss_fwd_kernel + ss_fixup_kernel) live in a fixed, file-scope device array.
//
// * Capacity: MWC_NOALLOC_SCRATCH_BYTES (4 MiB) per GPU, held by every GPU that loads this
//   library until the process exits. The segment planner keeps batch x channels x segments
//   below ~38K, i.e. at most ~2.6 MB of carries; a request that would need more is
//   rejected with MWC_ERR_UNSUPPORTED.
// * Set-up: the first call on each device, with that device current, looks up the array's
//   device address (cudaGetSymbolAddress) and keeps it; make that first call before any
//   stream capture.
// * Sharing: every call on a device uses the same array. Each call writes every carry it
//   reads, so nothing has to be cleared between calls, but calls that overlap on the GPU
//   (different streams, no ordering between them) race on the array.
// * Nothing here allocates: no cudaMalloc / cudaFree and no allocating library call.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "mwc_b200.h"
#include "mwc_device.cuh"
#include "mwc_internal.h"

using namespace mwc;

#define MWC_NOALLOC_SCRATCH_BYTES (4u << 20)

// The scratch itself: file scope, one copy per device that loads the library. In host code
// this name is only a stand-in; the kernels get the device address looked up below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MWC_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return report_error(MWC_ERR_CUDA, "cudaGetDevice failed");
    if (dev < 0 || dev >= kMaxDevices) return report_error(MWC_ERR_UNSUPPORTED, "device index out of range");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr) {
            char msg[256];
            snprintf(msg, sizeof(msg), "cudaGetSymbolAddress of the no-allocation scratch failed: %s",
                     cudaGetErrorString(e));
            return report_error(MWC_ERR_CUDA, msg);
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return MWC_OK;
}

bool aligned16_na(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" MWC_API int mwc_ss_fwd_noalloc(const void* u, const void* delta, const void* A,
                                          const void* Bm, const void* Cm, const void* Dv,
                                          const void* h_prev, void* out, void* h_last,
                                          float* ckpt, float* decay, int64_t B, int64_t L,
                                          int64_t D, int dtype, void* stream) {
    // the segmented kernels have no device waits: nothing for mwc_check_last_launch to read
    // (an earlier persistent call's error word may belong to a workspace already freed)
    note_err_word(nullptr);
    if (dtype != MWC_F32 && dtype != MWC_F16 && dtype != MWC_BF16)
        return report_error(MWC_ERR_INVALID, "u must be float32/float16/bfloat16");
    if (B < 0 || L < 0 || D < 0) return report_error(MWC_ERR_INVALID, "negative size");
    if (L == 0) return report_error(MWC_ERR_INVALID, "empty sequence (L=0)");
    if (B > 65535) return report_error(MWC_ERR_UNSUPPORTED, "batch exceeds 65535");
    if ((D + 3) / 4 > 0x7fffffffLL) return report_error(MWC_ERR_UNSUPPORTED, "D too large");
    if (!u || !delta || !A || !Bm || !Cm || !Dv)
        return report_error(MWC_ERR_INVALID, "u, delta, A, B_ssm, C_ssm and D_ssm are required");
    if (!out && !h_last && !ckpt && !decay) return report_error(MWC_ERR_INVALID, "no output requested");
    if (B == 0 || D == 0) return report_ok();

    const FwdPlan plan = plan_fwd(B, L, D, dtype, current_device_sms());
    const int64_t need = fwd_carry_floats(plan, B, D) * 4;
    if (need > (int64_t)MWC_NOALLOC_SCRATCH_BYTES) {
        char msg[256];
        snprintf(msg, sizeof(msg),
                 "no-allocation forward needs %lld bytes of scratch; it holds at most %u bytes",
                 (long long)need, MWC_NOALLOC_SCRATCH_BYTES);
        return report_error(MWC_ERR_UNSUPPORTED, msg);
    }
    void* scratch = nullptr;
    if (need > 0) {
        const int rc = scratch_address(&scratch);
        if (rc != MWC_OK) return rc;
    }

    const size_t es = dtype == MWC_F32 ? 4 : 2;
    FwdArgs a{};
    a.u = u; a.delta = delta; a.A = A; a.Bm = Bm; a.Cm = Cm; a.Dv = Dv;
    a.h_prev = h_prev; a.out = out; a.h_last = h_last; a.ckpt = ckpt; a.decay = decay;
    a.carry = plan.nseg > 1 ? static_cast<float*>(scratch) : nullptr;
    a.B = B; a.L = L; a.D = D;
    a.seg_len = plan.seg_len; a.nseg = plan.nseg;
    a.nck = (int)((L + CK - 1) / CK);
    a.vec = ((D * (int64_t)es) % 16 == 0) && aligned16_na(u) && aligned16_na(delta) &&
            (!out || aligned16_na(out));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = launch_fwd(a, plan, dtype, s);
    if (e != cudaSuccess) return report_error(MWC_ERR_CUDA, cudaGetErrorString(e));
    if (plan.nseg > 1) {
        FixupArgs f{};
        f.delta = delta; f.A = A; f.Cm = Cm; f.carry = a.carry;
        f.out = out; f.h_last = h_last; f.decay_out = decay; f.ckpt = ckpt;
        f.B = B; f.L = L; f.D = D; f.seg_len = plan.seg_len; f.nseg = plan.nseg;
        f.nck = a.nck; f.mode = 0; f.vec = a.vec;
        e = launch_fixup(f, plan, dtype, s);
        if (e != cudaSuccess) return report_error(MWC_ERR_CUDA, cudaGetErrorString(e));
    }
    return report_ok();
}
