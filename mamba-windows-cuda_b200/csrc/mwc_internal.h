// Host-side launch interface between the C ABI (capi.cu) and the kernel files.
#pragma once

#include <atomic>

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mwc {

// Forward scan over one L-segment per blockIdx.z (segment length seg_len, a multiple
// of the time tile). Segment 0 starts from h_prev (or 0), later segments from 0.
struct FwdArgs {
    const void* u;
    const void* delta;
    const void* A;
    const void* Bm;
    const void* Cm;
    const void* Dv;
    const void* h_prev;   // nullable
    void* out;            // nullable (checkpoint-only recompute)
    void* h_last;         // nullable; written only when nseg == 1
    float* ckpt;          // nullable; (B, nck, D, 16)
    float* decay;         // nullable; written only when nseg == 1
    float* carry;         // (B, nseg, D, 17) when nseg > 1: local end state + sum of delta
    int64_t B, L, D;
    int64_t seg_len;
    int nseg;
    int nck;
    int vec;              // 16-byte vector access of (.., D) rows is legal
    int N;                // states per channel: 0 or 16 (the reference's N), 32, 64
};

// Carry fold + truncated fixup. mode 0: h_in for segment s = 1 + blockIdx.z is folded from
// `carry`; mode 1: one segment over all of L with the explicit h_in / decay; mode 2: as mode 1,
// with L cut into chunks of FX_CHUNK_TILES 32-step tiles (blockIdx.z), each started from its
// delta prefix (dpre) and skipped when the incoming state has decayed below 2^-40 throughout.
struct FixupArgs {
    const void* delta;
    const void* A;
    const void* Cm;
    const float* carry;   // mode 0
    const float* h_in;    // modes 1 / 2
    const float* decay;   // modes 1 / 2 (needed for h_last)
    const float* dpre;    // mode 2: the forward's per-tile delta prefix records (PFwdArgs::dpre)
    void* out;            // nullable, read-modify-write
    void* h_last;         // nullable
    float* decay_out;     // nullable, mode 0: total decay of the call
    float* ckpt;          // nullable, read-modify-write
    int64_t B, L, D;
    int64_t seg_len;
    int nseg;
    int nck;
    int mode;
    int vec;
    int N;                // states per channel: 0 or 16 (the reference's N), 32, 64
};

struct BwdArgs {
    const void* u;
    const void* delta;
    const void* A;
    const void* Bm;
    const void* Cm;
    const void* Dv;
    const void* h_prev;   // nullable
    const void* dout;
    const void* dh_last;  // nullable
    const float* ckpt;    // required when nck > 1
    void* du;
    void* ddelta;
    void* dh_prev;        // nullable
    float* ws_bc;         // (nblk, B, nck*16, 32) per-CTA dB|dC partial sums
    float* ws_a;          // (B, D, 16) per-batch dA partial sums
    float* ws_d;          // (B, D) per-batch dD partial sums
    int64_t B, L, D;
    int nck;
    int nblk;
    int vec;
    int carry32;          // h_prev, dh_last, dh_prev are float32 (B, D, 16), not the I/O type
};

struct BwdFinalArgs {
    const float* ws_bc;
    const float* ws_a;
    const float* ws_d;
    void* dA;
    void* dB;
    void* dC;
    void* dD;
    int64_t B, L, D;
    int nck;
    int nblk;
};

struct LinArgs {
    const void* a;
    const void* x;     // fwd
    const void* h;     // bwd: forward output
    const void* g;     // bwd: upstream gradient
    void* out_h;       // fwd output
    void* ga;          // bwd outputs
    void* gx;
    int64_t R, L, N;
    int vec;
};

// Persistent TMA forward (ss_fwd_tma.cu). Tensor maps are 3-D (inner, L, B) views.
struct PFwdArgs {
    CUtensorMap tm_u, tm_d, tm_B, tm_C, tm_y;
    const void* A;
    const void* Dv;
    const void* h_prev;
    void* h_last;
    float* ckpt;
    float* decay;
    // nullable (launches with decay, modes 0 / 2): (B, ntiles, D, 2) float32, per 32-step tile
    // and channel the delta prefix sum before the tile and the minimum over the tile's steps
    // of the prefix sum through each step; the sequence-sharding fixup uses it to skip the
    // part of a range where the incoming state has decayed away
    float* dpre;
    float* hand;     // (chains, K, 128, 17): state + sum(delta) handed to the next unit
                     // (mode 0: record c of chain c, written by the head of a cut chain)
    int* flags;      // (chains, K) unit-done flags (mode 0: flag c)
    int* counter;    // unit queue head (mode 0: run index, in the order the CTAs start)
    int* err;        // bounded-wait error word
    int B, L, D;
    int nblk, nchains, K, seg_tiles, ntiles, nck;
    int has_out;
    int G, cpg;      // B / C groups (B_ssm, C_ssm are (B, L, G, 16)) and channels per group
    // 0: chained: one run of the chains' concatenated tiles per CTA; the tail of a chain cut
    //    between two runs waits for the record the head publishes;
    // 1: state only: segments 0..K-2 scan independently (segment 0 from h_prev, the others
    //    from zero) and each writes its end state and delta sum as its record;
    // 2: seeded: the records already hold each segment's incoming state and delta prefix sum
    //    (written by the fold kernel), so no segment waits or publishes.
    int mode;
};

struct PersistPlan {
    bool ok;        // chained: enough chains (>= SMs) for one run per SM; split: segments fit
    int nblk, nchains, ntiles, K, seg_tiles, grid;
};

PersistPlan plan_persistent(int64_t B, int64_t L, int64_t D, int num_sms);
int64_t persistent_ws_bytes(const PersistPlan& pl);
// Few (batch, 128-channel) chains: K independent segments per chain for the state-only /
// fold / seeded passes (ok = false when the shape has too few tiles for that).
PersistPlan plan_persistent_split(int64_t B, int64_t L, int64_t D, int num_sms);
cudaError_t launch_fwd_persistent_split(PFwdArgs& a, const PersistPlan& pl, int dtype, void* ws,
                                        cudaStream_t s);
bool make_tmap_3d(CUtensorMap* map, const void* base, int dtype, int64_t W, int64_t L, int64_t B,
                  int bw, int bl);
cudaError_t launch_fwd_persistent(PFwdArgs& a, const PersistPlan& pl, int dtype, void* ws,
                                  cudaStream_t s);

// Persistent TMA backward (ss_bwd_tma.cu).
struct PBwdArgs {
    CUtensorMap tm_u, tm_d, tm_g, tm_B, tm_C, tm_du, tm_dd;
    const void* A;
    const void* Dv;
    const void* h_prev;
    const void* dh_last;
    const float* ckpt;
    void* du;
    void* ddelta;
    void* dh_prev;
    float* hand;     // (chains, K, 128, 16): adjoint state handed to the previous segment
    float* ws_a;     // (units, 128, 16) dA partial sums
    float* ws_d;     // (units, 128) dD partial sums
    float* ws_bc;    // (B, nck*16, blocks, 32) dB | dC partial sums
    int* flags;
    int* counter;
    int* err;
    int B, L, D;
    int nblk, nchains, K, seg_tiles, ntiles, nck;
    int G, cpg;      // B / C groups (B_ssm, C_ssm, dB, dC are (B, L, G, 16)), channels per group
    // 0: chained segments (segment k waits for the adjoint state segment k+1 publishes);
    // 2: seeded: the records already hold the adjoint state at each segment's end (written
    //    by the adjoint-only pass and its fold), so no segment waits or publishes.
    int mode;
    int carry32;     // h_prev, dh_last, dh_prev are float32 (B, D, 16), not the I/O type
};

struct BwdPersistWs {
    int64_t off_hand, off_a, off_d, off_bc, off_sum, total;
};

PersistPlan plan_persistent_bwd(int64_t B, int64_t L, int64_t D, int num_sms);
BwdPersistWs bwd_persistent_ws(const PersistPlan& pl, int64_t B, int64_t L);
// Few chains: K independent segments per chain for the adjoint-only / fold / seeded passes.
PersistPlan plan_persistent_bwd_split(int64_t B, int64_t L, int64_t D, int num_sms);
cudaError_t launch_bwd_persistent_split(PBwdArgs& a, const PersistPlan& pl, int dtype, void* ws,
                                        const void* delta, const void* dout, const void* Cm,
                                        void* dA, void* dB, void* dC, void* dD, cudaStream_t s);
// Segment count for the few-chain split passes: the K (2..ntiles/min_seg) minimising
// waves x segment length, plus a small per-segment term; 0 when no K fits.
int pick_split_segments(int nchains, int ntiles, int num_sms, int min_seg_tiles);
cudaError_t launch_bwd_persistent(PBwdArgs& a, const PersistPlan& pl, int dtype, void* ws,
                                  void* dA, void* dB, void* dC, void* dD, cudaStream_t s);

// Error reporting shared by the C entry points (capi.cu).
int report_error(int code, const char* msg);
int report_ok();
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device): the attribute
// persists in the context, and setting it on every launch costs a driver call.
template <auto Kern>
inline cudaError_t ensure_smem_attr(int bytes) {
    static std::atomic<int> done[64];   // bytes already allowed, per device ordinal
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const bool cached = dev >= 0 && dev < 64;
    if (cached && done[dev].load(std::memory_order_relaxed) >= bytes) return cudaSuccess;
    e = cudaFuncSetAttribute(Kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && cached) done[dev].store(bytes, std::memory_order_relaxed);
    return e;
}

// Error word that mwc_check_last_launch reads for the last launch on this thread (nullptr: none).
void note_err_word(const int* word);
int current_device_sms();

// Launch-shape descriptors chosen by the host heuristics in capi.cu.
struct FwdPlan {
    int states_per_thread;  // 16, 8 or 4
    int channels_per_block;
    int nseg;
    int64_t seg_len;
};

FwdPlan plan_fwd(int64_t B, int64_t L, int64_t D, int dtype, int num_sms);
int64_t fwd_carry_floats(const FwdPlan& plan, int64_t B, int64_t D, int N = 16);
int bwd_channels_per_block(int dtype);

cudaError_t launch_fwd(const FwdArgs& a, const FwdPlan& plan, int dtype, cudaStream_t s);
cudaError_t launch_fixup(const FixupArgs& a, const FwdPlan& plan, int dtype, cudaStream_t s);
cudaError_t launch_bwd(const BwdArgs& a, int dtype, cudaStream_t s);
cudaError_t launch_bwd_final(const BwdFinalArgs& a, int dtype, cudaStream_t s);
cudaError_t launch_lin_fwd(const LinArgs& a, int dtype, cudaStream_t s);
// Adjoint at the start of a time range (ss_adjoint.cu): ws holds 2 x B x chunks x D x 16 floats.
int64_t adjoint_seq_chunks(int64_t L);
cudaError_t launch_adjoint_seq(const void* delta, const void* A, const void* Cm, const void* dout,
                               const float* q_in, float* q_out, float* ws, int64_t B, int64_t L, int64_t D,
                               int dtype, cudaStream_t s);
cudaError_t launch_lin_bwd(const LinArgs& a, int dtype, cudaStream_t s);

// One CTA waits on an mbarrier nothing arrives at, with a short bounded limit; records
// ERR_WAIT_TMA in *err and returns (selftest.cu).
cudaError_t launch_wait_selftest(int* err, cudaStream_t s);

}  // namespace mwc
