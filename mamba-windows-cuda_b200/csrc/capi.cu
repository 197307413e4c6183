// extern "C" entry points of libmwc_b200.so (declared in include/mwc_b200.h).
//
// Each entry point validates its arguments (messages follow the reference's TORCH_CHECK
// wording, mamba_windows_cuda/mamba_cuda.py:186-238), carves the caller's workspace,
// picks a launch plan for the current device and enqueues the kernels on the given stream.
// Nothing is allocated here and nothing blocks the host.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include <algorithm>

#include "mwc_b200.h"
#include "mwc_device.cuh"
#include "mwc_internal.h"
#include "mwc_tma.cuh"

using namespace mwc;

#define MWC_XSTR(x) #x
#define MWC_STR(x) MWC_XSTR(x)

namespace {

thread_local char g_err[512] = "";
// error word of the last persistent launch on this thread (nullptr: nothing to check)
thread_local const int* g_last_err_word = nullptr;

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int ok() {
    g_err[0] = '\0';
    return MWC_OK;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(MWC_ERR_CUDA, "%s: %s (%s)", where, cudaGetErrorName(e), cudaGetErrorString(e));
}

int device_sms() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
        n = 148;
    if (dev >= 0 && dev < 64) cache[dev] = n;
    return n;
}

size_t elem_size(int dtype) { return dtype == MWC_F32 ? 4 : 2; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Workspace layout of the backward: [ws_bc | ws_a | ws_d], each 256-byte aligned.
struct BwdWs {
    int64_t nblk, off_a, off_d, total;
};

BwdWs bwd_ws(int64_t B, int64_t L, int64_t D, int dtype) {
    BwdWs w;
    const int64_t cpb = bwd_channels_per_block(dtype);
    const int64_t nck = (L + CK - 1) / CK;
    w.nblk = (D + cpb - 1) / cpb;
    const int64_t bc = w.nblk * B * nck * CK * 2 * NSTATE * 4;
    w.off_a = align_up(bc, 256);
    w.off_d = align_up(w.off_a + B * D * NSTATE * 4, 256);
    w.total = align_up(w.off_d + B * D * 4, 256);
    return w;
}

int check_dtype(int dtype) {
    if (dtype != MWC_F32 && dtype != MWC_F16 && dtype != MWC_BF16)
        return fail(MWC_ERR_INVALID, "u must be float32/float16/bfloat16 (dtype code %d)", dtype);
    return MWC_OK;
}

int check_sizes(int64_t B, int64_t L, int64_t D) {
    if (B < 0 || L < 0 || D < 0)
        return fail(MWC_ERR_INVALID, "negative size (B=%lld, L=%lld, D=%lld)", (long long)B,
                    (long long)L, (long long)D);
    if (L == 0) return fail(MWC_ERR_INVALID, "empty sequence (L=0)");
    if (B > 65535) return fail(MWC_ERR_UNSUPPORTED, "batch %lld exceeds 65535", (long long)B);
    if ((D + 3) / 4 > 0x7fffffffLL) return fail(MWC_ERR_UNSUPPORTED, "D too large");
    return MWC_OK;
}

}  // namespace

namespace mwc {
// Error reporting for entry points defined in other files of the library.
int report_error(int code, const char* msg) {
    snprintf(g_err, sizeof(g_err), "%s", msg);
    return code;
}
int report_ok() { return ok(); }
void note_err_word(const int* word) { g_last_err_word = word; }
int current_device_sms() { return device_sms(); }
}  // namespace mwc

extern "C" {

int mwc_abi_version(void) { return MWC_ABI_VERSION; }

const char* mwc_last_error(void) { return g_err; }

const char* mwc_build_info(void) {
    return "libmwc_b200: sm_100a, CUDA " MWC_STR(__CUDACC_VER_MAJOR__) "." MWC_STR(
        __CUDACC_VER_MINOR__);
}

int64_t mwc_ss_ckpt_count(int64_t L) { return L <= 0 ? 0 : (L + CK - 1) / CK; }

int64_t mwc_ss_fwd_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype) {
    if (B <= 0 || L <= 0 || D <= 0) return 0;
    const int sms = device_sms();
    const FwdPlan plan = plan_fwd(B, L, D, dtype, sms);
    int64_t need = align_up(fwd_carry_floats(plan, B, D) * 4, 256);
    PersistPlan pp = plan_persistent(B, L, D, sms);
    if (!pp.ok) pp = plan_persistent_split(B, L, D, sms);
    if (pp.ok) need = std::max<int64_t>(need, align_up(persistent_ws_bytes(pp), 256));
    return need;
}

// B / C groups: G = 1 is the reference's (B, L, 16) layout; G > 1 gives (B, L, G, 16) with
// channel d in group d / (D / G), supported on the persistent paths when D / G is a
// multiple of the 128-channel block.
static int check_groups(int64_t D, int64_t G) {
    if (G < 1 || D % G != 0) return fail(MWC_ERR_INVALID, "groups must divide D (D=%lld, G=%lld)",
                                         (long long)D, (long long)G);
    if (G > 1 && (D / G) % 128 != 0)
        return fail(MWC_ERR_UNSUPPORTED, "grouped B / C need D / G to be a multiple of 128 (D=%lld, G=%lld)",
                    (long long)D, (long long)G);
    return MWC_OK;
}

static int fail_groups_path() {
    return fail(MWC_ERR_UNSUPPORTED,
                "grouped B / C run on the persistent path only: 16-byte-aligned buffers, rows of "
                "D x element size a multiple of 16 bytes, and at least as many (batch, 128-channel) "
                "chains as SMs or L >= 512");
}

static int ss_fwd_impl(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
                       const void* Dv, const void* h_prev, void* out, void* h_last, float* ckpt,
                       float* decay, void* workspace, int64_t workspace_bytes, int64_t B, int64_t L,
                       int64_t D, int64_t G, int dtype, void* stream, float* dpre = nullptr) {
    g_last_err_word = nullptr;
    int rc;
    if ((rc = check_dtype(dtype)) != MWC_OK) return rc;
    if ((rc = check_sizes(B, L, D)) != MWC_OK) return rc;
    if ((rc = check_groups(D, G)) != MWC_OK) return rc;
    if (!u || !delta || !A || !Bm || !Cm || !Dv)
        return fail(MWC_ERR_INVALID, "u, delta, A, B_ssm, C_ssm and D_ssm are required");
    if (!out && !h_last && !ckpt && !decay)
        return fail(MWC_ERR_INVALID, "no output requested");
    if (dpre && !decay) return fail(MWC_ERR_INVALID, "dprefix needs the decay output");
    if (B == 0 || D == 0) return ok();
    const int sms = device_sms();
    const size_t es0 = elem_size(dtype);
    // many (batch, 128-channel) chains: chained segments; few chains: state-only pass, fold,
    // seeded pass over independent L-segments
    const PersistPlan pchain = plan_persistent(B, L, D, sms);
    const bool split = !pchain.ok;
    const PersistPlan pp = split ? plan_persistent_split(B, L, D, sms) : pchain;
    const bool tma_ok = pp.ok && ((D * (int64_t)es0) % 16 == 0) && aligned16(u) &&
                        aligned16(delta) && aligned16(Bm) && aligned16(Cm) && aligned16(A) &&
                        aligned16(Dv) && (!h_prev || aligned16(h_prev)) &&
                        (!out || aligned16(out)) && L <= 0x7fffffffLL && D <= 0x7fffffffLL;
    if (tma_ok) {
        const int64_t pneed = align_up(persistent_ws_bytes(pp), 256);
        if (!workspace || workspace_bytes < pneed)
            return fail(MWC_ERR_WORKSPACE, "forward workspace of %lld bytes required, got %lld",
                        (long long)pneed, (long long)workspace_bytes);
        if (!aligned16(workspace))
            return fail(MWC_ERR_WORKSPACE, "forward workspace must be 16-byte aligned");
        PFwdArgs pa{};
        bool maps = make_tmap_3d(&pa.tm_u, u, dtype, D, L, B, 128, 32) &&
                    make_tmap_3d(&pa.tm_d, delta, dtype, D, L, B, 128, 32) &&
                    make_tmap_3d(&pa.tm_B, Bm, dtype, G * NSTATE, L, B, NSTATE, 32) &&
                    make_tmap_3d(&pa.tm_C, Cm, dtype, G * NSTATE, L, B, NSTATE, 32) &&
                    make_tmap_3d(&pa.tm_y, out ? out : u, dtype, D, L, B, 128, 32);
        if (maps) {
            pa.G = (int)G; pa.cpg = (int)(D / G);
            pa.A = A; pa.Dv = Dv; pa.h_prev = h_prev; pa.h_last = h_last;
            pa.ckpt = ckpt; pa.decay = decay; pa.dpre = dpre;
            pa.B = (int)B; pa.L = (int)L; pa.D = (int)D;
            pa.nck = (int)mwc_ss_ckpt_count(L);
            pa.has_out = out != nullptr;
            cudaStream_t st = static_cast<cudaStream_t>(stream);
            cudaError_t e = split ? launch_fwd_persistent_split(pa, pp, dtype, workspace, st)
                                  : launch_fwd_persistent(pa, pp, dtype, workspace, st);
            if (e != cudaSuccess) return cuda_fail(e, "selective-scan persistent forward launch");
            g_last_err_word = pa.err;
            return ok();
        }
    }
    if (G > 1) return fail_groups_path();
    if (dpre)
        return fail(MWC_ERR_UNSUPPORTED,
                    "dprefix is produced on the persistent path only (16-byte-aligned buffers, rows of "
                    "D x element size a multiple of 16 bytes, and B*D/128 >= SM count or L >= 512)");
    const FwdPlan plan = plan_fwd(B, L, D, dtype, sms);
    const int64_t need = align_up(fwd_carry_floats(plan, B, D) * 4, 256);
    if (need > 0 && (!workspace || workspace_bytes < need))
        return fail(MWC_ERR_WORKSPACE, "forward workspace of %lld bytes required, got %lld",
                    (long long)need, (long long)workspace_bytes);
    const size_t es = elem_size(dtype);
    FwdArgs a{};
    a.u = u; a.delta = delta; a.A = A; a.Bm = Bm; a.Cm = Cm; a.Dv = Dv;
    a.h_prev = h_prev; a.out = out; a.h_last = h_last; a.ckpt = ckpt; a.decay = decay;
    a.carry = plan.nseg > 1 ? static_cast<float*>(workspace) : nullptr;
    a.B = B; a.L = L; a.D = D;
    a.seg_len = plan.seg_len; a.nseg = plan.nseg;
    a.nck = (int)mwc_ss_ckpt_count(L);
    a.vec = ((D * (int64_t)es) % 16 == 0) && aligned16(u) && aligned16(delta) &&
            (!out || aligned16(out));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = launch_fwd(a, plan, dtype, s);
    if (e != cudaSuccess) return cuda_fail(e, "selective-scan forward launch");
    if (plan.nseg > 1) {
        FixupArgs f{};
        f.delta = delta; f.A = A; f.Cm = Cm; f.carry = a.carry;
        f.out = out; f.h_last = h_last; f.decay_out = decay; f.ckpt = ckpt;
        f.B = B; f.L = L; f.D = D; f.seg_len = plan.seg_len; f.nseg = plan.nseg;
        f.nck = a.nck; f.mode = 0; f.vec = a.vec;
        e = launch_fixup(f, plan, dtype, s);
        if (e != cudaSuccess) return cuda_fail(e, "selective-scan segment fixup launch");
    }
    return ok();
}

int mwc_ss_fwd(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
               const void* Dv, const void* h_prev, void* out, void* h_last, float* ckpt,
               float* decay, void* workspace, int64_t workspace_bytes, int64_t B, int64_t L,
               int64_t D, int dtype, void* stream) {
    return ss_fwd_impl(u, delta, A, Bm, Cm, Dv, h_prev, out, h_last, ckpt, decay, workspace,
                       workspace_bytes, B, L, D, 1, dtype, stream);
}

int mwc_ss_fwd_seq(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
                   const void* Dv, const void* h_prev, void* out, void* h_last, float* ckpt, float* decay,
                   float* dprefix, void* workspace, int64_t workspace_bytes, int64_t B, int64_t L,
                   int64_t D, int dtype, void* stream) {
    return ss_fwd_impl(u, delta, A, Bm, Cm, Dv, h_prev, out, h_last, ckpt, decay, workspace,
                       workspace_bytes, B, L, D, 1, dtype, stream, dprefix);
}

int64_t mwc_ss_dprefix_count(int64_t L) { return L <= 0 ? 0 : (L + DPRE_LT - 1) / DPRE_LT; }

int mwc_ss_fwd_grouped(const void* u, const void* delta, const void* A, const void* Bm,
                       const void* Cm, const void* Dv, const void* h_prev, void* out, void* h_last,
                       float* ckpt, float* decay, void* workspace, int64_t workspace_bytes,
                       int64_t B, int64_t L, int64_t D, int64_t G, int dtype, void* stream) {
    return ss_fwd_impl(u, delta, A, Bm, Cm, Dv, h_prev, out, h_last, ckpt, decay, workspace,
                       workspace_bytes, B, L, D, G, dtype, stream);
}

int64_t mwc_ss_fwd_nstate_workspace_bytes(int64_t B, int64_t L, int64_t D, int64_t N, int dtype) {
    if (N == NSTATE) return mwc_ss_fwd_workspace_bytes(B, L, D, dtype);
    if (B <= 0 || L <= 0 || D <= 0 || (N != 32 && N != 64)) return 0;
    const FwdPlan plan = plan_fwd(B, L, D, dtype, device_sms());
    return align_up(fwd_carry_floats(plan, B, D, (int)N) * 4, 256);
}

int mwc_ss_fwd_nstate(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
                      const void* Dv, const void* h_prev, void* out, void* h_last, float* ckpt,
                      float* decay, void* workspace, int64_t workspace_bytes, int64_t B, int64_t L,
                      int64_t D, int64_t N, int dtype, void* stream) {
    if (N == NSTATE)
        return ss_fwd_impl(u, delta, A, Bm, Cm, Dv, h_prev, out, h_last, ckpt, decay, workspace,
                           workspace_bytes, B, L, D, 1, dtype, stream);
    g_last_err_word = nullptr;
    int rc;
    if (N != 32 && N != 64) return fail(MWC_ERR_UNSUPPORTED, "N must be 16, 32 or 64 (got %lld)", (long long)N);
    if ((rc = check_dtype(dtype)) != MWC_OK) return rc;
    if ((rc = check_sizes(B, L, D)) != MWC_OK) return rc;
    if (!u || !delta || !A || !Bm || !Cm || !Dv)
        return fail(MWC_ERR_INVALID, "u, delta, A, B_ssm, C_ssm and D_ssm are required");
    if (!out && !h_last && !ckpt && !decay)
        return fail(MWC_ERR_INVALID, "no output requested");
    if (B == 0 || D == 0) return ok();
    // N = 32 / 64 run on the generic kernels (channel split over N / S lanes)
    const FwdPlan plan = plan_fwd(B, L, D, dtype, device_sms());
    const int64_t need = align_up(fwd_carry_floats(plan, B, D, (int)N) * 4, 256);
    if (need > 0 && (!workspace || workspace_bytes < need))
        return fail(MWC_ERR_WORKSPACE, "forward workspace of %lld bytes required, got %lld",
                    (long long)need, (long long)workspace_bytes);
    if (need > 0 && !aligned16(workspace))
        return fail(MWC_ERR_WORKSPACE, "forward workspace must be 16-byte aligned");
    const size_t es = elem_size(dtype);
    FwdArgs a{};
    a.u = u; a.delta = delta; a.A = A; a.Bm = Bm; a.Cm = Cm; a.Dv = Dv;
    a.h_prev = h_prev; a.out = out; a.h_last = h_last; a.ckpt = ckpt; a.decay = decay;
    a.carry = plan.nseg > 1 ? static_cast<float*>(workspace) : nullptr;
    a.B = B; a.L = L; a.D = D;
    a.seg_len = plan.seg_len; a.nseg = plan.nseg;
    a.nck = (int)mwc_ss_ckpt_count(L);
    a.vec = ((D * (int64_t)es) % 16 == 0) && aligned16(u) && aligned16(delta) && (!out || aligned16(out));
    a.N = (int)N;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = launch_fwd(a, plan, dtype, s);
    if (e != cudaSuccess) return cuda_fail(e, "selective-scan forward launch");
    if (plan.nseg > 1) {
        FixupArgs f{};
        f.delta = delta; f.A = A; f.Cm = Cm; f.carry = a.carry;
        f.out = out; f.h_last = h_last; f.decay_out = decay; f.ckpt = ckpt;
        f.B = B; f.L = L; f.D = D; f.seg_len = plan.seg_len; f.nseg = plan.nseg;
        f.nck = a.nck; f.mode = 0; f.vec = a.vec; f.N = (int)N;
        e = launch_fixup(f, plan, dtype, s);
        if (e != cudaSuccess) return cuda_fail(e, "selective-scan segment fixup launch");
    }
    return ok();
}

int64_t mwc_ss_bwd_workspace_bytes(int64_t B, int64_t L, int64_t D, int dtype) {
    if (B <= 0 || L <= 0 || D <= 0) return 0;
    int64_t need = bwd_ws(B, L, D, dtype).total;
    PersistPlan pb = plan_persistent_bwd(B, L, D, device_sms());
    if (!pb.ok) pb = plan_persistent_bwd_split(B, L, D, device_sms());
    if (pb.ok) need = std::max<int64_t>(need, bwd_persistent_ws(pb, B, L).total);
    return need;
}

static int ss_bwd_impl(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
                       const void* Dv, const void* h_prev, const void* dout, const void* dh_last,
                       const float* ckpt, void* du, void* ddelta, void* dA, void* dB, void* dC, void* dD,
                       void* dh_prev, void* workspace, int64_t workspace_bytes, int64_t B, int64_t L,
                       int64_t D, int64_t G, int dtype, void* stream, bool carry32 = false) {
    g_last_err_word = nullptr;
    int rc;
    if ((rc = check_dtype(dtype)) != MWC_OK) return rc;
    if ((rc = check_sizes(B, L, D)) != MWC_OK) return rc;
    if ((rc = check_groups(D, G)) != MWC_OK) return rc;
    if (!u || !delta || !A || !Bm || !Cm || !Dv || !dout)
        return fail(MWC_ERR_INVALID, "u, delta, A, B_ssm, C_ssm, D_ssm and dout are required");
    if (!du || !ddelta || !dA || !dB || !dC || !dD)
        return fail(MWC_ERR_INVALID, "du, ddelta, dA, dB, dC and dD outputs are required");
    const int64_t nck = mwc_ss_ckpt_count(L);
    if (nck > 1 && !ckpt)
        return fail(MWC_ERR_INVALID, "checkpoint states are required when L > %d", CK);
    if (B == 0 || D == 0) return ok();
    {
        const size_t es0 = elem_size(dtype);
        // many chains: chained segments; few chains: adjoint-only pass, fold, seeded pass
        const PersistPlan pchain = plan_persistent_bwd(B, L, D, device_sms());
        const bool split = !pchain.ok;
        const PersistPlan pb = split ? plan_persistent_bwd_split(B, L, D, device_sms()) : pchain;
        const bool tma_ok = pb.ok && ((D * (int64_t)es0) % 16 == 0) && aligned16(u) &&
                            aligned16(delta) && aligned16(dout) && aligned16(Bm) &&
                            aligned16(Cm) && aligned16(A) && aligned16(du) && aligned16(ddelta) &&
                            (!ckpt || aligned16(ckpt)) && (!h_prev || aligned16(h_prev)) &&
                            (!dh_last || aligned16(dh_last)) && (!dh_prev || aligned16(dh_prev)) &&
                            L <= 0x7fffffffLL && D <= 0x7fffffffLL;
        if (tma_ok) {
            const BwdPersistWs pw = bwd_persistent_ws(pb, B, L);
            if (!workspace || workspace_bytes < pw.total)
                return fail(MWC_ERR_WORKSPACE, "backward workspace of %lld bytes required, got %lld",
                            (long long)pw.total, (long long)workspace_bytes);
            if (!aligned16(workspace))
                return fail(MWC_ERR_WORKSPACE, "backward workspace must be 16-byte aligned");
            PBwdArgs pa{};
            const bool maps = make_tmap_3d(&pa.tm_u, u, dtype, D, L, B, 128, CK) &&
                              make_tmap_3d(&pa.tm_d, delta, dtype, D, L, B, 128, CK) &&
                              make_tmap_3d(&pa.tm_g, dout, dtype, D, L, B, 128, CK) &&
                              make_tmap_3d(&pa.tm_B, Bm, dtype, G * NSTATE, L, B, NSTATE, CK) &&
                              make_tmap_3d(&pa.tm_C, Cm, dtype, G * NSTATE, L, B, NSTATE, CK) &&
                              make_tmap_3d(&pa.tm_du, du, dtype, D, L, B, 128, CK) &&
                              make_tmap_3d(&pa.tm_dd, ddelta, dtype, D, L, B, 128, CK);
            if (maps) {
                pa.A = A; pa.Dv = Dv; pa.h_prev = h_prev; pa.dh_last = dh_last; pa.ckpt = ckpt;
                pa.du = du; pa.ddelta = ddelta; pa.dh_prev = dh_prev;
                pa.B = (int)B; pa.L = (int)L; pa.D = (int)D; pa.nck = (int)nck;
                pa.G = (int)G; pa.cpg = (int)(D / G);
                pa.carry32 = carry32 ? 1 : 0;
                cudaStream_t st = static_cast<cudaStream_t>(stream);
                cudaError_t e = split ? launch_bwd_persistent_split(pa, pb, dtype, workspace, delta, dout, Cm,
                                                                    dA, dB, dC, dD, st)
                                      : launch_bwd_persistent(pa, pb, dtype, workspace, dA, dB, dC, dD, st);
                if (e != cudaSuccess) return cuda_fail(e, "selective-scan persistent backward launch");
                g_last_err_word = pa.err;
                return ok();
            }
        }
    }
    if (G > 1) return fail_groups_path();
    const BwdWs w = bwd_ws(B, L, D, dtype);
    if (!workspace || workspace_bytes < w.total)
        return fail(MWC_ERR_WORKSPACE, "backward workspace of %lld bytes required, got %lld",
                    (long long)w.total, (long long)workspace_bytes);
    if (!aligned16(workspace))
        return fail(MWC_ERR_WORKSPACE, "backward workspace must be 16-byte aligned");
    const size_t es = elem_size(dtype);
    char* ws = static_cast<char*>(workspace);
    BwdArgs a{};
    a.u = u; a.delta = delta; a.A = A; a.Bm = Bm; a.Cm = Cm; a.Dv = Dv;
    a.h_prev = h_prev; a.dout = dout; a.dh_last = dh_last; a.ckpt = ckpt;
    a.du = du; a.ddelta = ddelta; a.dh_prev = dh_prev;
    a.carry32 = carry32 ? 1 : 0;
    a.ws_bc = reinterpret_cast<float*>(ws);
    a.ws_a = reinterpret_cast<float*>(ws + w.off_a);
    a.ws_d = reinterpret_cast<float*>(ws + w.off_d);
    a.B = B; a.L = L; a.D = D; a.nck = (int)nck; a.nblk = (int)w.nblk;
    a.vec = ((D * (int64_t)es) % 16 == 0) && aligned16(u) && aligned16(delta) &&
            aligned16(dout) && aligned16(du) && aligned16(ddelta);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = launch_bwd(a, dtype, s);
    if (e != cudaSuccess) return cuda_fail(e, "selective-scan backward launch");
    BwdFinalArgs f{};
    f.ws_bc = a.ws_bc; f.ws_a = a.ws_a; f.ws_d = a.ws_d;
    f.dA = dA; f.dB = dB; f.dC = dC; f.dD = dD;
    f.B = B; f.L = L; f.D = D; f.nck = (int)nck; f.nblk = (int)w.nblk;
    e = launch_bwd_final(f, dtype, s);
    if (e != cudaSuccess) return cuda_fail(e, "selective-scan backward reduction launch");
    return ok();
}

int mwc_ss_bwd(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
               const void* Dv, const void* h_prev, const void* dout, const void* dh_last,
               const float* ckpt, void* du, void* ddelta, void* dA, void* dB, void* dC, void* dD,
               void* dh_prev, void* workspace, int64_t workspace_bytes, int64_t B, int64_t L,
               int64_t D, int dtype, void* stream) {
    return ss_bwd_impl(u, delta, A, Bm, Cm, Dv, h_prev, dout, dh_last, ckpt, du, ddelta, dA, dB, dC,
                       dD, dh_prev, workspace, workspace_bytes, B, L, D, 1, dtype, stream);
}

int mwc_ss_bwd_seq(const void* u, const void* delta, const void* A, const void* Bm, const void* Cm,
                   const void* Dv, const float* h_in, const void* dout, const float* q_in,
                   const float* ckpt, void* du, void* ddelta, void* dA, void* dB, void* dC, void* dD,
                   float* q_out, void* workspace, int64_t workspace_bytes, int64_t B, int64_t L,
                   int64_t D, int dtype, void* stream) {
    return ss_bwd_impl(u, delta, A, Bm, Cm, Dv, h_in, dout, q_in, ckpt, du, ddelta, dA, dB, dC, dD,
                       q_out, workspace, workspace_bytes, B, L, D, 1, dtype, stream, true);
}

int mwc_ss_bwd_grouped(const void* u, const void* delta, const void* A, const void* Bm,
                       const void* Cm, const void* Dv, const void* h_prev, const void* dout,
                       const void* dh_last, const float* ckpt, void* du, void* ddelta, void* dA,
                       void* dB, void* dC, void* dD, void* dh_prev, void* workspace,
                       int64_t workspace_bytes, int64_t B, int64_t L, int64_t D, int64_t G,
                       int dtype, void* stream) {
    return ss_bwd_impl(u, delta, A, Bm, Cm, Dv, h_prev, dout, dh_last, ckpt, du, ddelta, dA, dB, dC,
                       dD, dh_prev, workspace, workspace_bytes, B, L, D, G, dtype, stream);
}

int mwc_ss_plan(int64_t B, int64_t L, int64_t D, int dtype, int backward, int32_t* info) {
    int rc;
    if (info == nullptr) return fail(MWC_ERR_INVALID, "info (4 x int32) is required");
    if ((rc = check_dtype(dtype)) != MWC_OK) return rc;
    if ((rc = check_sizes(B, L, D)) != MWC_OK) return rc;
    info[0] = MWC_PATH_GENERIC;
    info[1] = info[2] = info[3] = 0;
    if (B == 0 || D == 0) return ok();
    const int sms = device_sms();
    const bool rows16 = (D * (int64_t)elem_size(dtype)) % 16 == 0 && L <= 0x7fffffffLL && D <= 0x7fffffffLL;
    PersistPlan pp = backward ? plan_persistent_bwd(B, L, D, sms) : plan_persistent(B, L, D, sms);
    int path = MWC_PATH_CHAINED;
    if (!pp.ok) {
        pp = backward ? plan_persistent_bwd_split(B, L, D, sms) : plan_persistent_split(B, L, D, sms);
        path = MWC_PATH_SPLIT;
    }
    if (pp.ok && rows16) {
        info[0] = path;
        info[1] = pp.K;
        info[2] = pp.seg_tiles;
        info[3] = pp.grid;
        return ok();
    }
    if (!backward) {
        const FwdPlan plan = plan_fwd(B, L, D, dtype, sms);
        info[1] = plan.nseg;
        info[2] = (int32_t)std::min<int64_t>(plan.seg_len, 0x7fffffff);
        info[3] = (int32_t)std::min<int64_t>(((D + plan.channels_per_block - 1) / plan.channels_per_block) * B *
                                                 plan.nseg, 0x7fffffff);
    } else {
        info[1] = 1;
        info[2] = (int32_t)std::min<int64_t>(L, 0x7fffffff);
        info[3] = (int32_t)std::min<int64_t>(bwd_ws(B, L, D, dtype).nblk * B, 0x7fffffff);
    }
    return ok();
}

int mwc_ss_fixup(const void* delta, const void* A, const void* Cm, const float* h_in,
                 const float* decay, void* out, void* h_last, float* ckpt, int64_t B, int64_t L,
                 int64_t D, int dtype, void* stream) {
    int rc;
    if ((rc = check_dtype(dtype)) != MWC_OK) return rc;
    if ((rc = check_sizes(B, L, D)) != MWC_OK) return rc;
    if (!delta || !A || !h_in) return fail(MWC_ERR_INVALID, "delta, A and h_in are required");
    if (out && !Cm) return fail(MWC_ERR_INVALID, "C_ssm is required to correct the output");
    if (h_last && !decay) return fail(MWC_ERR_INVALID, "decay is required to correct h_last");
    if (B == 0 || D == 0) return ok();
    FwdPlan plan = plan_fwd(B, L, D, dtype, device_sms());
    plan.nseg = 1;
    plan.seg_len = L;
    const size_t es = elem_size(dtype);
    FixupArgs f{};
    f.delta = delta; f.A = A; f.Cm = Cm; f.h_in = h_in; f.decay = decay;
    f.out = out; f.h_last = h_last; f.ckpt = ckpt;
    f.B = B; f.L = L; f.D = D; f.seg_len = L; f.nseg = 1;
    f.nck = (int)mwc_ss_ckpt_count(L); f.mode = 1;
    f.vec = ((D * (int64_t)es) % 16 == 0) && aligned16(delta) && (!out || aligned16(out));
    cudaError_t e = launch_fixup(f, plan, dtype, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "selective-scan fixup launch");
    return ok();
}

int64_t mwc_ss_adjoint_seq_workspace_bytes(int64_t B, int64_t L, int64_t D) {
    if (B <= 0 || L <= 0 || D <= 0) return 0;
    return 2 * B * adjoint_seq_chunks(L) * D * NSTATE * (int64_t)sizeof(float);
}

int mwc_ss_adjoint_seq(const void* delta, const void* A, const void* Cm, const void* dout, const float* q_in,
                       float* q_out, void* workspace, int64_t workspace_bytes, int64_t B, int64_t L,
                       int64_t D, int dtype, void* stream) {
    int rc;
    if ((rc = check_dtype(dtype)) != MWC_OK) return rc;
    if ((rc = check_sizes(B, L, D)) != MWC_OK) return rc;
    if (!delta || !A || !Cm || !dout || !q_out)
        return fail(MWC_ERR_INVALID, "delta, A, C_ssm, dout and q_out are required");
    if (B == 0 || D == 0) return ok();
    if (adjoint_seq_chunks(L) > 65535 || B > 65535)
        return fail(MWC_ERR_UNSUPPORTED, "sequence or batch too long for the range adjoint");
    const int64_t need = mwc_ss_adjoint_seq_workspace_bytes(B, L, D);
    if (!workspace || workspace_bytes < need)
        return fail(MWC_ERR_WORKSPACE, "range-adjoint workspace of %lld bytes required, got %lld",
                    (long long)need, (long long)workspace_bytes);
    if (!aligned16(workspace)) return fail(MWC_ERR_WORKSPACE, "range-adjoint workspace must be 16-byte aligned");
    cudaError_t e = launch_adjoint_seq(delta, A, Cm, dout, q_in, q_out, static_cast<float*>(workspace), B, L, D,
                                       dtype, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "range-adjoint launch");
    return ok();
}

int mwc_ss_fixup_chunked(const void* delta, const void* A, const void* Cm, const float* h_in,
                         const float* decay, const float* dprefix, void* out, void* h_last, float* ckpt,
                         int64_t B, int64_t L, int64_t D, int dtype, void* stream) {
    int rc;
    if ((rc = check_dtype(dtype)) != MWC_OK) return rc;
    if ((rc = check_sizes(B, L, D)) != MWC_OK) return rc;
    if (!delta || !A || !h_in || !dprefix)
        return fail(MWC_ERR_INVALID, "delta, A, h_in and dprefix are required");
    if (out && !Cm) return fail(MWC_ERR_INVALID, "C_ssm is required to correct the output");
    if (h_last && !decay) return fail(MWC_ERR_INVALID, "decay is required to correct h_last");
    if (B == 0 || D == 0) return ok();
    const int64_t chunk = (int64_t)FX_CHUNK_TILES * DPRE_LT;
    const int64_t nchunk = (L + chunk - 1) / chunk;
    if (nchunk > 65535) return fail(MWC_ERR_UNSUPPORTED, "sequence too long for the chunked fixup");
    FwdPlan plan = plan_fwd(B, L, D, dtype, device_sms());
    plan.nseg = (int)nchunk;
    plan.seg_len = chunk;
    const size_t es = elem_size(dtype);
    FixupArgs f{};
    f.delta = delta; f.A = A; f.Cm = Cm; f.h_in = h_in; f.decay = decay; f.dpre = dprefix;
    f.out = out; f.h_last = h_last; f.ckpt = ckpt;
    f.B = B; f.L = L; f.D = D; f.seg_len = chunk; f.nseg = (int)nchunk;
    f.nck = (int)mwc_ss_ckpt_count(L); f.mode = 2;
    f.vec = ((D * (int64_t)es) % 16 == 0) && aligned16(delta) && (!out || aligned16(out));
    cudaError_t e = launch_fixup(f, plan, dtype, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "selective-scan chunked fixup launch");
    return ok();
}

int mwc_lin_scan_fwd(const void* a, const void* x, void* h, int64_t R, int64_t L, int64_t N,
                     int dtype, void* stream) {
    int rc;
    if ((rc = check_dtype(dtype)) != MWC_OK) return rc;
    if (R < 0 || L < 0 || N < 0) return fail(MWC_ERR_INVALID, "negative size");
    if (!a || !x || !h) return fail(MWC_ERR_INVALID, "A, X and the output are required");
    if (R == 0 || L == 0 || N == 0) return ok();
    if ((R + 3) / 4 > 0x7fffffffLL || (N + 31) / 32 > 65535)
        return fail(MWC_ERR_UNSUPPORTED, "scan shape too large");
    const size_t es = elem_size(dtype);
    LinArgs la{};
    la.a = a; la.x = x; la.out_h = h; la.R = R; la.L = L; la.N = N;
    la.vec = (N == 1) && ((L * (int64_t)es) % 16 == 0) && aligned16(a) && aligned16(x) &&
             aligned16(h);
    cudaError_t e = launch_lin_fwd(la, dtype, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "linear scan forward launch");
    return ok();
}

int mwc_lin_scan_bwd(const void* a, const void* h, const void* g, void* ga, void* gx, int64_t R,
                     int64_t L, int64_t N, int dtype, void* stream) {
    int rc;
    if ((rc = check_dtype(dtype)) != MWC_OK) return rc;
    if (R < 0 || L < 0 || N < 0) return fail(MWC_ERR_INVALID, "negative size");
    if (!a || !h || !g || !ga || !gx)
        return fail(MWC_ERR_INVALID, "A, H, grad and both gradient outputs are required");
    if (R == 0 || L == 0 || N == 0) return ok();
    if ((R + 3) / 4 > 0x7fffffffLL || (N + 31) / 32 > 65535)
        return fail(MWC_ERR_UNSUPPORTED, "scan shape too large");
    LinArgs la{};
    la.a = a; la.h = h; la.g = g; la.ga = ga; la.gx = gx; la.R = R; la.L = L; la.N = N;
    la.vec = 0;
    cudaError_t e = launch_lin_bwd(la, dtype, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "linear scan backward launch");
    return ok();
}

int mwc_check_last_launch(void* stream) {
    const int* word = g_last_err_word;
    if (word == nullptr) return ok();
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "waiting for the stream");
    int code = 0;
    e = cudaMemcpy(&code, word, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "reading the device error word");
    if (code == 0) return ok();
    return fail(MWC_ERR_TIMEOUT, "a bounded device wait of the last persistent kernel gave up "
                "(code %d: %s); its results are invalid", code,
                code == ERR_WAIT_TMA ? "pipeline barrier" :
                code == ERR_WAIT_CHAIN ? "segment hand-off" :
                code == ERR_SMEM_ALIGN ? "shared memory alignment" : "unknown");
}

int mwc_selftest_wait_timeout(int* dev_word, void* stream) {
    if (dev_word == nullptr) return fail(MWC_ERR_INVALID, "dev_word is required");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(dev_word, 0, sizeof(int), s);
    if (e == cudaSuccess) e = launch_wait_selftest(dev_word, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    int code = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&code, dev_word, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "wait self-test");
    if (code == ERR_WAIT_TMA) return fail(MWC_ERR_TIMEOUT, "self-test wait expired as intended");
    return code == 0 ? ok() : fail(MWC_ERR_CUDA, "self-test recorded unexpected code %d", code);
}

}  // extern "C"
