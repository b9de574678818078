// K2: fused tiered decode attention for sm_100a.
//
// Replaces, for one decode step of one layer, the reference's
//   TieredKVCache._materialize (fade/cache.py:693-808: cat(sink, dequant(middle),
//   recent)) followed by HF SDPA (transformers sdpa_attention.py:40-62), and the
//   standalone fused_int4_sdpa (fade/kernels/fused_int4_attn.py:277-342).
// Attention is a sum over keys, so the tiers are processed independently and
// merged: the token order of the reference's cat() does not matter.
//
// Launch sequence (one stream, chained with programmatic dependent launch):
//   k0  rotate_queries   (only with a rotated tier): q_rot = q @ R^T in fp32,
//                        16 query rows per CTA, R^T staged in shared memory,
//                        a 2 x 4 register tile per thread.
//   k1  middle_kernel    one persistent CTA per SM, 16 warps:
//       * 3 consumer groups x 4 warps.  The CTA owns a contiguous range of
//         128-token units of the quantised middle (stream-K over all (b, kv-
//         head) rows); group g takes units g, g+3, ... of it.
//       * 3 producer warps (one per group): 2-D TMA (cp.async.bulk.tensor, no
//         multicast) of 128-byte swizzled rows of packed K and V codes, plus V
//         scales, into a ring of up to 12 stages with full/empty mbarriers.
//         With `early` (prefetch_tiers) they stream before the grid
//         dependency resolves.
//       * consumer warp = 32 tokens of a stage: ldmatrix -> exact code
//         conversion (shift + lop3 magic exponent, the LUT-free int4 -> half
//         conversion of FasterTransformer's mixed-precision GEMMs, then one
//         packed subtract) -> packed multiply by the scale, which rounds each
//         element exactly like the reference's rnd(q * scale) -> mma.sync
//         m16n8k16 in the model dtype (the GQA query rows are N) -> online
//         softmax in log2 space with lazy maxima -> movmatrix transposes P ->
//         O^T += V^T P^T.  2-bit rotated codes fold their scales exactly
//         (c * s is representable) into q and P.  At a row boundary the
//         group's 4 warps combine in shared memory in a fixed order and store
//         one partial (plain stores: no fences, counters or waits between CTAs).
//       * one FP-tier warp: attention over the sink / recent tokens of its rows
//         (all of them staged with one cp.async pass), P split hi + lo; with
//         the fused age-out it quantises the oldest ring token into the middle,
//         attends its INT4 round trip and the new token, and writes the new
//         token into the ring.
//       * every mbarrier wait is bounded; a stalled pipeline sets the
//         workspace error word (fade_workspace_check) instead of hanging.
//   k1' middle_tc_kernel (middle_tc.cuh; opt-in with fade_set_middle_kernel,
//                        INT4 K/V at D = 128): the same schedule and partials
//                        with tcgen05 MMAs and tensor-memory accumulators.
//   k2  finish_kernel    one CTA per (b, kv-head), after the middle grid: merge
//                        of the FP partial with the row's middle partials (the
//                        rotation R applied back for rotated tiers), normalise,
//                        write `out`, advance the age-out lengths.  Without a
//                        quantised tier it computes the FP tiers itself.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace fade {

constexpr int kConsumerWarps = 4;  // per consumer group; 32 tokens of a stage each
constexpr int kStageTokens = 128;  // 32 tokens per consumer warp
static_assert(kStageTokens == FADE_PAGE_TOKENS, "a page of a paged middle is one streaming unit");
// One middle CTA per SM: G consumer groups (3 for up to 8 query rows per kv
// head; 1 above, where the wider state needs the registers) share one
// producer warp and one ring of stages; group g
// consumes stages g, g+G, g+2G, ...
__host__ __device__ constexpr int mid_groups(int NT) { return NT == 1 ? 3 : 1; }
// + one producer warp per group + the FP-tier warp
__host__ __device__ constexpr int mid_threads(int NT) {
    return (mid_groups(NT) * (kConsumerWarps + 1) + 1) * 32;
}
constexpr int kMidMaxStages = 15;
constexpr int kFpChunk = 80;       // FP-tier tokens the FP warp stages per pass (sink + recent + new)
constexpr int kSmemPerBlock = 232448;  // 227 KB opt-in shared memory per CTA
constexpr float kLog2e = 1.4426950408889634f;
// Initial running maximum of the middle kernel's online softmax: finite and
// below any real score, so exp2(score - max) never sees inf - inf.
constexpr float kMaskedMax = -1e30f;
constexpr uint32_t kWaitPolls = 1u << 15;   // bounded mbarrier polling ...
constexpr uint32_t kWaitHintNs = 10000;   // ... of up to 10 us each

// ---------------------------------------------------------------------------
// PTX wrappers (mbarrier, TMA, ldmatrix, movmatrix, mma)
// ---------------------------------------------------------------------------
// Non-blocking test of a phase.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait that lets the hardware suspend the warp up to `ns` nanoseconds
// until the phase completes (fewer polling instructions while waiting)
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}
// Bounded wait: gives up after kWaitLimit polls (each poll may suspend the
// thread for a hardware-defined interval) and never spins forever.  A CTA-wide
// abort flag makes every later wait of the CTA fail at once, so a CTA whose
// pipeline stalled walks the rest of its (uniform) control flow quickly and
// exits; the device error word tells the host.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err) {
    if (mbar_try_wait(bar, parity)) return true;   // common case: one poll
    if (*abort_flag) return false;
    // each poll suspends up to kWaitHintNs: at most kWaitPolls * kWaitHintNs
    // (about 0.3 s) in total, then the CTA aborts
    for (uint32_t i = 0; i < kWaitPolls; ++i) {
        if (mbar_try_wait_hint(bar, parity, kWaitHintNs)) return true;
        if ((i & 63u) == 63u && *abort_flag) return false;
    }
    *abort_flag = 1;
    atomicExch(err, 1);
    return false;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void tma_load_1d(uint32_t dst, const CUtensorMap* map, int x, uint32_t bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.1d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2}], [%3], %4;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t addr, uint32_t (&r)[2]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t a) {
    uint32_t d;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
    return d;
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// ---------------------------------------------------------------------------
// Model-dtype packed math (f16x2 / bf16x2) and the MMA in the model dtype.
// ---------------------------------------------------------------------------
template <int DT> struct Pk;
template <> struct Pk<FADE_F16> {
    __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ __forceinline__ static float unpack_lo(uint32_t v) {
        return __half2float(__ushort_as_half((unsigned short)(v & 0xFFFFu)));
    }
    // magic exponent: (x & 0xF) ^ 0x6408 = fp16(1024 + u), u = nibble ^ 8 = code + 8
    static constexpr uint32_t K4 = 0x64086408u, B4 = 0x64086408u;   // bias 1032
    static constexpr uint32_t K2 = 0x64026402u, B2 = 0x64026402u;   // bias 1026
    __device__ __forceinline__ static void mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
};
template <> struct Pk<FADE_BF16> {
    __device__ __forceinline__ static uint32_t sub(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t mul(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ __forceinline__ static float unpack_lo(uint32_t v) { return __uint_as_float(v << 16); }
    // bf16(128 + u): exponent of 128, 7 mantissa bits hold u in 0..15
    static constexpr uint32_t K4 = 0x43084308u, B4 = 0x43084308u;   // bias 136
    static constexpr uint32_t K2 = 0x43024302u, B2 = 0x43024302u;   // bias 130
    __device__ __forceinline__ static void mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
            "{%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
};

// ---------------------------------------------------------------------------
// Code -> exact model-dtype integers ("LUT-free" magic-exponent conversion, as
// in FasterTransformer's mixed-precision GEMMs): every field is shifted to the
// low bits, (x & mask) ^ K forms the float 2^k + (code + bias) with the sign
// bit of the two's-complement field flipped (offset binary), and one packed
// subtraction of 2^k + bias leaves the code exactly.  The caller then
// multiplies by the scale with one packed multiply, which rounds exactly like
// the reference's `q.to(dtype) * scale.to(dtype)` (fade/quant.py:124-127).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t shr_k(uint32_t x, int i) { return x >> (4 * (i + 1)); }
__device__ __forceinline__ uint32_t hfma2_f16(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
template <int DT> struct Conv {
    // INT4: bytes b0..b3 of x hold elements (2j: high nibble, 2j+1: low).
    // h[0]=(e1,e5) h[1]=(e0,e4) h[2]=(e3,e7) h[3]=(e2,e6)
    // fp16: the nibbles at bits 4-7 / 20-23 need no shift: masked in place
    // they read fp16(1024 + 16 u) and one packed FMA (v / 16 - 72, exact)
    // leaves the code, so 8 codes take one shift instead of three.  bf16 has
    // too few mantissa bits for that and shifts every field down.
    __device__ __forceinline__ static void int4(uint32_t x, uint32_t (&h)[4]) {
        if constexpr (DT == FADE_F16) {
            const uint32_t y = x >> 8;
            h[0] = Pk<DT>::sub(lop3_and_xor(x, 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
            h[1] = hfma2_f16(lop3_and_xor(x, 0x00F000F0u, 0x64806480u), 0x2C002C00u, 0xD480D480u);
            h[2] = Pk<DT>::sub(lop3_and_xor(y, 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
            h[3] = hfma2_f16(lop3_and_xor(y, 0x00F000F0u, 0x64806480u), 0x2C002C00u, 0xD480D480u);
        } else {
            h[0] = Pk<DT>::sub(lop3_and_xor(x, 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
            h[1] = Pk<DT>::sub(lop3_and_xor(shr_k(x, 0), 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
            h[2] = Pk<DT>::sub(lop3_and_xor(shr_k(x, 1), 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
            h[3] = Pk<DT>::sub(lop3_and_xor(shr_k(x, 2), 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
        }
    }
    // 2-bit: field f of a byte sits at bit 6-2f.  h[0..3] = fields 3,2,1,0 of
    // bytes (0,2); h[4..7] = fields 3,2,1,0 of bytes (1,3).
    __device__ __forceinline__ static void int2(uint32_t x, uint32_t (&h)[8]) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            h[i] = Pk<DT>::sub(lop3_and_xor(x >> (2 * i), 0x00030003u, Pk<DT>::K2), Pk<DT>::B2);
    }
    // bf16, biased and scaled by powers of 4: fields 3, 2, 1 of a byte are
    // masked where they lie (bits 0-1, 2-3, 4-5 sit inside the 7 mantissa
    // bits of bf16(128 + m)), field 0 (bits 6-7) is shifted down.  h[i] holds
    // the same fields as int2() but as the exact value F * (code + 2) + 128,
    // F = 1, 4, 16, 1 for fields 3, 2, 1, 0 (the channel's kF2 factor), so a
    // word of 16 codes takes 3 shifts + 8 lop3 instead of 8 + 8.
    // fp16 (ten mantissa bits): all four fields of a byte lie inside the
    // mantissa of fp16(1024 + m), so only the odd bytes are shifted: 16 codes
    // take 1 shift + 8 lop3; h[i] = F * (code + 2) + 1024 with F = 1, 4, 16,
    // 64 for fields 3, 2, 1, 0 (kF2h).
    __device__ __forceinline__ static void int2_biased(uint32_t x, uint32_t (&h)[8]) {
        if constexpr (DT == FADE_F16) {
            const uint32_t y = x >> 8;
            h[0] = lop3_and_xor(x, 0x00030003u, 0x64026402u);
            h[1] = lop3_and_xor(x, 0x000C000Cu, 0x64086408u);
            h[2] = lop3_and_xor(x, 0x00300030u, 0x64206420u);
            h[3] = lop3_and_xor(x, 0x00C000C0u, 0x64806480u);
            h[4] = lop3_and_xor(y, 0x00030003u, 0x64026402u);
            h[5] = lop3_and_xor(y, 0x000C000Cu, 0x64086408u);
            h[6] = lop3_and_xor(y, 0x00300030u, 0x64206420u);
            h[7] = lop3_and_xor(y, 0x00C000C0u, 0x64806480u);
            return;
        }
        const uint32_t y = x >> 8;
        h[0] = lop3_and_xor(x, 0x00030003u, 0x43024302u);
        h[1] = lop3_and_xor(x, 0x000C000Cu, 0x43084308u);
        h[2] = lop3_and_xor(x, 0x00300030u, 0x43204320u);
        h[3] = lop3_and_xor(x >> 6, 0x00030003u, 0x43024302u);
        h[4] = lop3_and_xor(y, 0x00030003u, 0x43024302u);
        h[5] = lop3_and_xor(y, 0x000C000Cu, 0x43084308u);
        h[6] = lop3_and_xor(y, 0x00300030u, 0x43204320u);
        h[7] = lop3_and_xor(x >> 14, 0x00030003u, 0x43024302u);
    }
};

// Channel d of a 2-bit row is field d % 4 of its byte; int2_biased() returns
// it as kF2(d) * code + kH2(d) (kH2 = 128 + 2 * kF2).
__host__ __device__ constexpr float kF2(int d) { return (d & 3) == 1 ? 16.f : (d & 3) == 2 ? 4.f : 1.f; }
__host__ __device__ constexpr float kInvF2(int d) { return (d & 3) == 1 ? 0.0625f : (d & 3) == 2 ? 0.25f : 1.f; }
__host__ __device__ constexpr float kH2(int d) { return 128.f + 2.f * kF2(d); }
// The fp16 form (Conv<FADE_F16>::int2_biased): field 0 (d % 4 == 0) is read in
// place as F = 64; kH2h = 1024 + 2 * kF2h.
__host__ __device__ constexpr float kF2h(int d) { return (d & 3) == 0 ? 64.f : kF2(d); }
__host__ __device__ constexpr float kInvF2h(int d) { return (d & 3) == 0 ? 0.015625f : kInvF2(d); }
__host__ __device__ constexpr float kH2h(int d) { return 1024.f + 2.f * kF2h(d); }

// ---------------------------------------------------------------------------
// Channel maps.  For the K operand, k-step ks and slot s in {0,1,2,3} (= the
// A/B fragment k indices 2t, 2t+1, 2t+8, 2t+9) of thread t = lane % 4,
// kdim() is the channel.  For the V operand (O^T rows), m-tile mi and row half
// hr (0: row gid, 1: row gid+8), gid = lane / 4, vdim() is the channel.
// The orders follow the conversion outputs above, so no data is shuffled.
// ---------------------------------------------------------------------------
template <int BITS> struct ChanMap;
template <> struct ChanMap<4> {
    __device__ __forceinline__ static int kdim(int ks, int s, int t) {
        const int cb = ks >> 1, u = ks & 1;
        const int off[2][4] = {{1, 5, 0, 4}, {3, 7, 2, 6}};
        return 32 * cb + 8 * t + off[u][s];
    }
    __device__ __forceinline__ static int vdim(int mi, int hr, int gid) {
        const int cb = mi >> 1, j = mi & 1;
        return 32 * cb + 4 * gid + 2 * j + hr;
    }
};
template <> struct ChanMap<2> {
    __device__ __forceinline__ static int kdim(int ks, int s, int t) {
        const int cb = ks >> 2, u = ks & 3;
        const int off[4][4] = {{3, 11, 2, 10}, {1, 9, 0, 8}, {7, 15, 6, 14}, {5, 13, 4, 12}};
        return 64 * cb + 16 * t + off[u][s];
    }
    __device__ __forceinline__ static int vdim(int mi, int hr, int gid) {
        const int cb = mi >> 2, j = mi & 3;
        return 64 * cb + 8 * gid + 2 * j + hr;
    }
};

// ---------------------------------------------------------------------------
// Kernel parameters
// ---------------------------------------------------------------------------
struct FpSeg {
    const void* k;
    const void* v;
    int64_t row_sb, row_sh;
    const int64_t* row_base;
    const int32_t* lens;
    int64_t len;
};

struct MidParams {
    int dtype;
    int B, Hq, Hkv, D, n_q, g, rows;
    float qk_scale;                 // sm_scale * log2(e)
    const void* q;                  // dtype [B,Hq,n_q,D] (strided) or fp32 q_rot
    int64_t q_sb, q_sh, q_ss;
    int q_is_f32;                   // 1: q points at the fp32 rotated queries
    const void* k_scale;            // per-channel, dtype
    int64_t ks_sb, ks_sh;
    const void* v_scale;            // per-token (row-indexed) or grouped
    int group;                      // grouped V: tokens per group, else 0
    int64_t row_sb, row_sh;
    const int64_t* row_base;
    const int32_t* lens;
    int64_t len;
    const int32_t* cu_units;        // ragged: [Z+1]; null = uniform
    const int32_t* page_table;      // paged middle: [Z][pages_per_row] page ids, or null
    int64_t pages_per_row;
    int units_per_z;                // uniform case
    int n_ctas;
    float* ws_ml;                   // [U][rows][2] partial (max, sum), log2 domain
    float* ws_o;                    // [U][rows][D] un-normalised partial output
    int* ws_err;
    int scale_tma;                  // V scales arrive by TMA (row starts 8-aligned)
    int q_vec;                      // q / k_scale rows allow 16-byte loads
    int early;                      // producer may stream before the previous kernel ends
    // FP tiers (the FP warp): segments, the model-dtype query, partial outputs
    int n_fp;
    FpSeg fp[FADE_MAX_SEGMENTS];
    const void* qo;                 // dtype [B,Hq,n_q,D]
    int64_t qo_sb, qo_sh, qo_ss;
    float* ws_fpml;                 // [Z][rows][2]
    float* ws_fpo;                  // [Z][rows][D]
    // fused age-out (fade_decode_attn_age_out), age == 0 otherwise
    int age;
    int ring_fp;                    // index into fp[] of the recent-window ring
    int64_t ring_cap, ring_origin;
    const void* k_new;              // [B,Hkv,D]
    const void* v_new;
    int64_t new_sb, new_sh;
    int64_t mid_cap;
    const int32_t* mid_len;         // = lens
    uint8_t* age_k;                 // = the middle's code rows, written at row n
    uint8_t* age_v;
    int* ws_age;                    // [Z] middle length after the step
};

__device__ __forceinline__ int64_t seg_len(const MidParams& p, int b) {
    return p.lens ? (int64_t)p.lens[b] : p.len;
}
__device__ __forceinline__ int64_t seg_row0(const MidParams& p, int z) {
    const int b = z / p.Hkv, h = z % p.Hkv;
    return p.row_base ? p.row_base[z] : (int64_t)b * p.row_sb + (int64_t)h * p.row_sh;
}
__device__ __forceinline__ int total_units(const MidParams& p, int Z) {
    return p.cu_units ? p.cu_units[Z] : Z * p.units_per_z;
}
__device__ __forceinline__ int units_begin(const MidParams& p, int z) {
    return p.cu_units ? p.cu_units[z] : z * p.units_per_z;
}
// z such that units_begin(z) <= u < units_begin(z+1)
__device__ __forceinline__ int z_of_unit(const MidParams& p, int Z, int u) {
    if (!p.cu_units) return u / p.units_per_z;
    int lo = 0, hi = Z - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (p.cu_units[mid] <= u) lo = mid; else hi = mid - 1;
    }
    return lo;
}
__device__ __forceinline__ int cta_of_unit(int u, int C, int U) {
    return (int)(((int64_t)(u + 1) * C - 1) / U);
}

template <int D, int KB, int VB, bool VGROUP, int NT>
struct MidLayout {
    static constexpr int RBK = D * KB / 8;
    static constexpr int RBV = D * VB / 8;
    static constexpr int NCHK = RBK / 16;
    static constexpr int NCHV = RBV / 16;
    static constexpr int K_BYTES = kStageTokens * RBK;
    static constexpr int V_BYTES = kStageTokens * RBV;
    // scale region: per-token V scales or grouped V scales [groups][D], raw
    // dtype bits, for up to kStageTokens/16 groups.
    static constexpr int SC_BYTES = VGROUP ? (kStageTokens / 16) * D * 2 : kStageTokens * 2;
    // bytes the scale TMA box of one stage carries (grouped: kStageTokens/G groups)
    __host__ __device__ static constexpr int sc_box_bytes(int group) {
        return VGROUP ? (kStageTokens / group) * D * 2 : kStageTokens * 2;
    }
    // [K0 V0 K1 V1 ...] (each region a multiple of 1024 B, so every TMA
    // destination keeps the 1024-B alignment the swizzle modes need), then
    // the per-stage scale regions.
    static constexpr int K_OFF = 0;
    static constexpr int V_OFF = K_BYTES;
    static constexpr int STAGE_BYTES = K_BYTES + V_BYTES;
    static_assert(K_BYTES % 1024 == 0 && V_BYTES % 1024 == 0, "stage regions must stay 1 KB aligned");
    static constexpr int G = mid_groups(NT);
    static constexpr int ML_BYTES = 2 * kConsumerWarps * NT * 8 * 2 * 4;  // per group: per-warp row stats, 2 buffers
    // as many stages as shared memory holds (a multiple of G, so each ring
    // slot always serves the same group)
    static constexpr int AB_BYTES = 2 * kFpChunk * (D + 8) * 2;   // FP warp: staged K and V rows
    static constexpr int NS_FIT = (kSmemPerBlock - 1024 - 16 - AB_BYTES - 2 * kMidMaxStages * 8 -
                                   G * ML_BYTES) /
                                  (STAGE_BYTES + SC_BYTES);
    static constexpr int NS = ((NS_FIT < kMidMaxStages ? NS_FIT : kMidMaxStages) / G) * G;
    static_assert(NS >= 2 * G, "shared memory too small for the stage ring");
    static constexpr int SC_BASE = NS * STAGE_BYTES;
    static constexpr int RING_BYTES = SC_BASE + NS * SC_BYTES;
    static constexpr int BAR_OFF = RING_BYTES + G * ML_BYTES;
    static constexpr int FLAG_OFF = BAR_OFF + 2 * NS * 8;
    static constexpr int AB_OFF = FLAG_OFF + 16;
    static constexpr int SMEM_BYTES = AB_OFF + AB_BYTES + 1024;  // +1024 for alignment
    static_assert(SMEM_BYTES <= kSmemPerBlock, "middle kernel shared memory over the per-CTA limit");
};


template <int DT>
__device__ __forceinline__ float load_f(const void* p, int64_t i) {
    return Elem<DT>::to_f(reinterpret_cast<const typename Elem<DT>::T*>(p)[i]);
}
template <int DT>
__device__ __forceinline__ uint16_t load_bits(const void* p, int64_t i) {
    return reinterpret_cast<const uint16_t*>(p)[i];
}

__device__ __forceinline__ uint32_t dup16(uint16_t v) { return (uint32_t)v | ((uint32_t)v << 16); }

// Load the 2*NCH ldmatrix tiles (token block tb, 16-byte chunk cb) of one
// 16-token m-tile: r[tb][cb].  TRANS selects the transposing form (V).
// Stage tiles hold packed token rows of NCH*16 bytes, 128/(NCH*16) tokens per
// 128-byte shared-memory row, swizzled by the TMA unit's 128B pattern
// (16-byte chunk c of row R lands at chunk c ^ (R & 7)): every 8-row ldmatrix
// read below touches 8 distinct bank groups.
template <int NCH>
__device__ __forceinline__ uint32_t tile_off(int tok, int cb) {
    constexpr int TPR = 8 / NCH;  // tokens per 128-byte row
    const int row = tok / TPR;
    const int chunk = (tok % TPR) * NCH + cb;
    return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// Per-lane shared-memory offsets of the ldmatrix reads of a warp's two
// 16-token m-tiles, computed once per kernel.  When an m-tile step moves the
// swizzle rows by a multiple of 8 the second m-tile is the first plus a
// constant (the XOR pattern repeats every 8 rows).
template <int NCH>
struct TileOffs {
    static constexpr int TPR = 8 / NCH;
    static constexpr int NX = (2 * NCH >= 4) ? 2 * NCH / 4 : 1;
    static constexpr bool SHIFT = ((16 / TPR) % 8) == 0;
    static constexpr uint32_t MT_STEP = (16 / TPR) * 128;
    uint32_t o[SHIFT ? 1 : 2][NX];
    __device__ __forceinline__ TileOffs(int trow_warp, int lane) {
#pragma unroll
        for (int mt = 0; mt < (SHIFT ? 1 : 2); ++mt)
#pragma unroll
            for (int x = 0; x < NX; ++x) {
                const int trow0 = trow_warp + mt * 16;
                if constexpr (2 * NCH >= 4) {
                    const int mi = x * 4 + lane / 8;
                    o[mt][x] = tile_off<NCH>(trow0 + (mi / NCH) * 8 + (lane & 7), mi % NCH);
                } else {
                    o[mt][x] = tile_off<NCH>(trow0 + ((lane / 8) & 1) * 8 + (lane & 7), 0);
                }
            }
    }
    __device__ __forceinline__ uint32_t get(int mt, int x) const {
        if constexpr (SHIFT) return o[0][x] + (uint32_t)mt * MT_STEP;
        else return o[mt][x];
    }
};

template <int NCH, bool TRANS>
__device__ __forceinline__ void load_tiles_at(uint32_t base, const TileOffs<NCH>& to, int mt,
                                              uint32_t (&r)[2][NCH]) {
    constexpr int NMAT = 2 * NCH;
    if constexpr (NMAT >= 4) {
#pragma unroll
        for (int x = 0; x < NMAT / 4; ++x) {
            uint32_t r4[4];
            if constexpr (TRANS) ldsm_x4_t(base + to.get(mt, x), r4);
            else ldsm_x4(base + to.get(mt, x), r4);
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                const int mj = x * 4 + y;
                r[mj / NCH][mj % NCH] = r4[y];
            }
        }
    } else {
        uint32_t r2[2];
        if constexpr (TRANS) ldsm_x2_t(base + to.get(mt, 0), r2);
        else ldsm_x2(base + to.get(mt, 0), r2);
        r[0][0] = r2[0];
        r[1][0] = r2[1];
    }
}

template <int NCH, bool TRANS>
__device__ __forceinline__ void load_tiles(uint32_t base, int trow0, int lane, uint32_t (&r)[2][NCH]) {
    constexpr int NMAT = 2 * NCH;
    if constexpr (NMAT >= 4) {
#pragma unroll
        for (int x = 0; x < NMAT / 4; ++x) {
            const int mi = x * 4 + lane / 8;
            const int tb = mi / NCH, cb = mi % NCH;
            const uint32_t off = tile_off<NCH>(trow0 + tb * 8 + (lane & 7), cb);
            uint32_t r4[4];
            if constexpr (TRANS) ldsm_x4_t(base + off, r4);
            else ldsm_x4(base + off, r4);
#pragma unroll
            for (int y = 0; y < 4; ++y) {
                const int mj = x * 4 + y;
                r[mj / NCH][mj % NCH] = r4[y];
            }
        }
    } else {
        const int tb = (lane / 8) & 1;
        const uint32_t off = tile_off<NCH>(trow0 + tb * 8 + (lane & 7), 0);
        uint32_t r2[2];
        if constexpr (TRANS) ldsm_x2_t(base + off, r2);
        else ldsm_x2(base + off, r2);
        r[0][0] = r2[0];
        r[1][0] = r2[1];
    }
}

// ---------------------------------------------------------------------------
// FP-tier warp of the middle kernel (one per CTA): attention over the FP
// tiers (sinks, recent window) of the rows z in [c*Z/n, (c+1)*Z/n), written as
// one un-normalised partial per row for the finisher, while the consumer
// groups stream the middle.  The FP tokens of a row are staged into shared
// memory with 16-byte cp.async in chunks of kFpChunk tokens (one memory round
// trip per chunk, so the warp's latency stays well below the streaming time),
// then multiplied with ldmatrix + mma.sync like the consumer path.  With the
// fused age-out the warp also moves the oldest ring token into the middle
// (INT4 codes exactly as fade_age_out_int4): its staged row is replaced by
// the INT4 round trip, the step's new token is staged after the FP tokens,
// and the new token is written into the freed ring slot.
// ---------------------------------------------------------------------------
template <int DT, int D, int NT>
__device__ __forceinline__ void fp_rows_warp_body(const MidParams& p, int c, int n_cta, uint8_t* fsm, bool waited) {
    using T = typename Elem<DT>::T;
    using P = Pk<DT>;
    constexpr int KSTEPS = D / 16, MT = D / 16;
    constexpr int RS = D + 8;                // padded smem row (elements): conflict-free ldmatrix
    constexpr int PCS = D / 8;               // 16-byte pieces per row
    constexpr int DPL = D / 32;              // channels per lane in the age-out
    const int lane = threadIdx.x % 32, gid = lane >> 2, t = lane & 3;
    const int Z = p.B * p.Hkv;
    const int z0 = (int)((int64_t)c * Z / n_cta), z1 = (int)((int64_t)(c + 1) * Z / n_cta);
    T* ksm = reinterpret_cast<T*>(fsm);
    T* vsm = ksm + kFpChunk * RS;
    for (int z = z0; z < z1; ++z) {
        const int b = z / p.Hkv, h = z % p.Hkv;
        // ---- FP segments of the row ----
        int64_t sl[FADE_MAX_SEGMENTS], sr[FADE_MAX_SEGMENTS], T_seg = 0;
#pragma unroll
        for (int s = 0; s < FADE_MAX_SEGMENTS; ++s) {
            sl[s] = 0;
            sr[s] = 0;
            if (s < p.n_fp) {
                sl[s] = p.fp[s].lens ? (int64_t)p.fp[s].lens[b] : p.fp[s].len;
                sr[s] = p.fp[s].row_base ? p.fp[s].row_base[z] : (int64_t)b * p.fp[s].row_sb + (int64_t)h * p.fp[s].row_sh;
                T_seg += sl[s];
            }
        }
        // ---- fused age-out bookkeeping (the middle length is read below,
        //      together with the first chunk's copies: one memory round trip) ----
        int64_t n = 0, ft_aged = -1, slot = 0;
        bool room = false;
        // the step's new token is staged after the FP tokens whenever an
        // age-out runs, and attended only when the middle has room
        const int64_t T_stage = T_seg + (p.age ? 1 : 0);
        int64_t T_all = T_seg;
        float scpre[DPL];
#pragma unroll
        for (int i = 0; i < DPL; ++i) scpre[i] = 0.f;
        const T* kn = reinterpret_cast<const T*>(p.k_new) + (int64_t)b * p.new_sb + (int64_t)h * p.new_sh;
        const T* vn = reinterpret_cast<const T*>(p.v_new) + (int64_t)b * p.new_sb + (int64_t)h * p.new_sh;
        // ---- query fragments (exact model-dtype q), natural channel order;
        //      loaded after the grid dependency resolves ----
        uint32_t qf[NT][KSTEPS][2];
        auto load_q = [&]() {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int r = nt * 8 + gid;
                const bool rv = r < p.rows;
                const int j = rv ? r / p.n_q : 0, sq = rv ? r % p.n_q : 0;
                const uint32_t* qp = reinterpret_cast<const uint32_t*>(
                    reinterpret_cast<const T*>(p.qo) + (int64_t)b * p.qo_sb + (int64_t)(h * p.g + j) * p.qo_sh +
                    (int64_t)sq * p.qo_ss);
#pragma unroll
                for (int ks = 0; ks < KSTEPS; ++ks) {
                    qf[nt][ks][0] = rv ? qp[ks * 8 + t] : 0u;       // channels 16ks + 2t, +1
                    qf[nt][ks][1] = rv ? qp[ks * 8 + 4 + t] : 0u;   // channels 16ks + 2t + 8, +9
                }
            }
        };
        float m_run[NT][2], l_run[NT][2], o[NT][MT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m_run[nt][0] = m_run[nt][1] = kMaskedMax;
            l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
            for (int mi = 0; mi < MT; ++mi)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[nt][mi][e] = 0.f;
        }
        for (int64_t c0 = 0; c0 < T_stage; c0 += kFpChunk) {
            const int nc = (int)((T_stage - c0) < kFpChunk ? (T_stage - c0) : kFpChunk);
            const int nc16 = (nc + 15) & ~15;
            __syncwarp();   // the previous chunk's rows are no longer read
            // ---- stage K and V rows (padding rows up to a multiple of 16: row 0).
            //      The cache tiers first; the step's new token (written by the
            //      preceding kernel) only after the grid dependency resolves. ----
            auto stage = [&](bool new_token) {
                for (int i = lane; i < nc16 * PCS; i += 32) {
                    const int tk = i / PCS, pc = i % PCS;
                    int64_t ft = c0 + (tk < nc ? tk : 0);
                    if ((ft >= T_seg) != new_token) continue;
                    const T* ks;
                    const T* vs;
                    if (ft >= T_seg) {
                        ks = kn + pc * 8;
                        vs = vn + pc * 8;
                    } else {
                        int s = 0;
                        while (s < p.n_fp - 1 && ft >= sl[s]) { ft -= sl[s]; ++s; }
                        const int64_t off = (sr[s] + ft) * D + pc * 8;
                        ks = reinterpret_cast<const T*>(p.fp[s].k) + off;
                        vs = reinterpret_cast<const T*>(p.fp[s].v) + off;
                    }
                    cp_async16(smem_u32(ksm + tk * RS + pc * 8), ks);
                    cp_async16(smem_u32(vsm + tk * RS + pc * 8), vs);
                }
            };
            stage(false);
            if (c0 == 0 && p.age) {
                // loads in flight with the copies above
                n = p.mid_len[b];
                const T* ksc = reinterpret_cast<const T*>(p.k_scale) + (int64_t)b * p.ks_sb + (int64_t)h * p.ks_sh;
#pragma unroll
                for (int i = 0; i < DPL; ++i) scpre[i] = Elem<DT>::to_f(ksc[lane * DPL + i]);
                room = n < p.mid_cap;
                if (room) {
                    slot = (n - p.ring_origin) % p.ring_cap;
                    if (slot < 0) slot += p.ring_cap;
                    ft_aged = slot;
                    for (int s = 0; s < p.ring_fp; ++s) ft_aged += sl[s];
                    T_all = T_seg + 1;
                }
            }
            if (!waited) {
                griddep_wait();
                waited = true;
            }
            stage(true);
            if (c0 == 0) {
                load_q();
                if (p.age && lane == 0) p.ws_age[z] = (int)(room ? n + 1 : n);
            }
            cp_async_wait_all();
            __syncwarp();
            if (ft_aged >= c0 && ft_aged < c0 + nc) {
                // ---- the aged token: INT4 codes into the middle, its staged row
                //      becomes rnd(code * scale); the new token takes its ring slot ----
                T* kr = ksm + (ft_aged - c0) * RS;
                T* vr = vsm + (ft_aged - c0) * RS;
                float kx[DPL], vx[DPL], sc[DPL];
#pragma unroll
                for (int i = 0; i < DPL; ++i) {
                    const int d = lane * DPL + i;
                    kx[i] = Elem<DT>::to_f(kr[d]);
                    vx[i] = Elem<DT>::to_f(vr[d]);
                    sc[i] = scpre[i];
                }
                float m = 0.f;
#pragma unroll
                for (int i = 0; i < DPL; ++i) m = fmaxf(m, fabsf(vx[i]));
#pragma unroll
                for (int o2 = 16; o2 > 0; o2 >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o2));
                m = fmaxf(m, Elem<DT>::eps());
                const float inv = inv_scale<DT>(m, 7.f);
                const float vsc = Elem<DT>::rnd(__fdiv_rn(m, 7.f));
                const int64_t mrow = (p.row_base ? p.row_base[z] : (int64_t)b * p.row_sb + (int64_t)h * p.row_sh) + n;
                if (lane == 0) reinterpret_cast<T*>(const_cast<void*>(p.v_scale))[mrow] = Elem<DT>::from_f(vsc);
#pragma unroll
                for (int i = 0; i < DPL; i += 2) {
                    int kq[2], vq[2];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const int d = lane * DPL + i + j;
                        kq[j] = (sc[i + j] > 0.f) ? quant_code(__fdiv_rn(kx[i + j], sc[i + j]), -8.f, 7.f) : 0;
                        vq[j] = quant_code(Elem<DT>::rnd(__fmul_rn(vx[i + j], inv)), -8.f, 7.f);
                        kr[d] = Elem<DT>::from_f((float)kq[j] * sc[i + j]);
                        vr[d] = Elem<DT>::from_f((float)vq[j] * vsc);
                    }
                    const int pp = (lane * DPL + i) / 2;
                    p.age_k[mrow * (D / 2) + pp] = (uint8_t)(((kq[0] & 15) << 4) | (kq[1] & 15));
                    p.age_v[mrow * (D / 2) + pp] = (uint8_t)(((vq[0] & 15) << 4) | (vq[1] & 15));
                }
                // ring slot <- new token (this lane's channels; the old row was staged above)
                T* rk = reinterpret_cast<T*>(const_cast<void*>(p.fp[p.ring_fp].k)) + (sr[p.ring_fp] + slot) * D;
                T* rv = reinterpret_cast<T*>(const_cast<void*>(p.fp[p.ring_fp].v)) + (sr[p.ring_fp] + slot) * D;
#pragma unroll
                for (int i = 0; i < DPL; ++i) {
                    const int d = lane * DPL + i;
                    rk[d] = kn[d];
                    rv[d] = vn[d];
                }
                __syncwarp();
            }
            // ---- attention over the chunk, 16 tokens per m-tile ----
            const uint32_t kbase = smem_u32(ksm), vbase = smem_u32(vsm);
            const int lrow = (lane & 7) + ((lane >> 3) & 1) * 8, lcol = (lane >> 4) * 8;       // K (A) tiles
            const int vrow = (lane & 7) + (lane >> 4) * 8, vcol = ((lane >> 3) & 1) * 8;       // V^T (A) tiles
            for (int t0 = 0; t0 < nc16; t0 += 16) {
                float sacc[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) sacc[nt][e] = 0.f;
#pragma unroll
                for (int ks = 0; ks < KSTEPS; ++ks) {
                    uint32_t a[4];
                    ldsm_x4(kbase + (uint32_t)(((t0 + lrow) * RS + ks * 16 + lcol) * 2), a);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) P::mma(sacc[nt], a[0], a[1], a[2], a[3], qf[nt][ks][0], qf[nt][ks][1]);
                }
                // ---- online softmax (log2 domain); padding rows masked ----
                bool grow = false;
                float corr[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int tk = t0 + gid + ((e >> 1) << 3);
                        sacc[nt][e] = (c0 + tk >= T_all) ? -INFINITY : sacc[nt][e] * p.qk_scale;
                    }
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        float mx = fmaxf(sacc[nt][e], sacc[nt][e + 2]);
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                        const float mnew = fmaxf(m_run[nt][e], mx);
                        grow |= mnew > m_run[nt][e];
                        corr[nt][e] = ex2(m_run[nt][e] - mnew);
                        m_run[nt][e] = mnew;
                    }
                }
                if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            l_run[nt][e] *= corr[nt][e];
#pragma unroll
                            for (int mi = 0; mi < MT; ++mi) {
                                o[nt][mi][e] *= corr[nt][e];
                                o[nt][mi][e + 2] *= corr[nt][e];
                            }
                        }
                }
                // P as hi + lo model-dtype parts (two MMAs): the FP tiers carry
                // the sharpest scores, so P keeps ~16 significant bits here
                uint32_t pb[NT][2], pl[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    float pv[4], lo[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        pv[e] = ex2(sacc[nt][e] - m_run[nt][e & 1]);
                        l_run[nt][e & 1] += pv[e];
                    }
                    const uint32_t h01 = P::pack(pv[0], pv[1]), h23 = P::pack(pv[2], pv[3]);
                    lo[0] = pv[0] - P::unpack_lo(h01);
                    lo[1] = pv[1] - P::unpack_lo(h01 >> 16);
                    lo[2] = pv[2] - P::unpack_lo(h23);
                    lo[3] = pv[3] - P::unpack_lo(h23 >> 16);
                    pb[nt][0] = movmatrix_t(h01);
                    pb[nt][1] = movmatrix_t(h23);
                    pl[nt][0] = movmatrix_t(P::pack(lo[0], lo[1]));
                    pl[nt][1] = movmatrix_t(P::pack(lo[2], lo[3]));
                }
                // ---- O^T += V^T . P^T (V^T fragments by transposing ldmatrix) ----
#pragma unroll
                for (int mi = 0; mi < MT; ++mi) {
                    uint32_t a[4];
                    ldsm_x4_t(vbase + (uint32_t)(((t0 + vrow) * RS + mi * 16 + vcol) * 2), a);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        P::mma(o[nt][mi], a[0], a[1], a[2], a[3], pb[nt][0], pb[nt][1]);
                        P::mma(o[nt][mi], a[0], a[1], a[2], a[3], pl[nt][0], pl[nt][1]);
                    }
                }
            }
        }
        if (!waited) {   // no FP token: the workspace is written only after the dependency
            griddep_wait();
            waited = true;
        }
        if (T_stage == 0 && p.age && lane == 0) p.ws_age[z] = (int)n;
        // ---- partial of row z: O^T rows are channels mi*16 + gid (+8) ----
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float l = l_run[nt][e];
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                const int r = nt * 8 + 2 * t + e;
                if (r < p.rows) {
                    if (gid == 0)
                        *reinterpret_cast<float2*>(p.ws_fpml + ((int64_t)z * p.rows + r) * 2) =
                            make_float2(m_run[nt][e], l);
                    float* dst = p.ws_fpo + ((int64_t)z * p.rows + r) * D;
#pragma unroll
                    for (int mi = 0; mi < MT; ++mi) {
                        dst[mi * 16 + gid] = o[nt][mi][e];
                        dst[mi * 16 + gid + 8] = o[nt][mi][e + 2];
                    }
                }
            }
        __syncwarp();
    }
}

// The FP-tier warp as a call of its own in the mma.sync middle kernel (keeps
// that kernel's register allocation unchanged); the tcgen05 kernel inlines
// the body, where a call would keep its arrays in local memory.
template <int DT, int D, int NT>
__device__ __noinline__ void fp_rows_warp(const MidParams& p, int c, int n_cta, uint8_t* fsm, bool waited) {
    fp_rows_warp_body<DT, D, NT>(p, c, n_cta, fsm, waited);
}


// ---------------------------------------------------------------------------
// k1: middle tier, persistent stream-K
// QSPLIT: the query is fp32 (rotated tiers) and is fed to the MMA as a
// hi + lo pair of model-dtype values (two MMAs per k-step).
// ---------------------------------------------------------------------------
template <int DT, int D, int KB, int VB, bool VGROUP, int NT, bool QSPLIT>
__global__ void __launch_bounds__(mid_threads(NT), 1)
middle_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
              const __grid_constant__ CUtensorMap tmap_s, const __grid_constant__ MidParams p) {
    using L = MidLayout<D, KB, VB, VGROUP, NT>;
    using KMap = ChanMap<KB>;
    using VMap = ChanMap<VB>;
    using P = Pk<DT>;
    constexpr int KSTEPS = D / 16;   // k-steps of the QK product
    constexpr int MT = D / 16;       // m-tiles of the PV product (rows = channels)
    // 2-bit codes c in {-2,-1,0,1}: c * scale is exactly representable, so the
    // reference's rnd(c * scale) equals c * scale and the scales can be folded
    // exactly: K's per-channel scale into the fp32 query (before its hi + lo
    // split), V's per-token scale into P.  The codes enter the MMA as is.
    constexpr bool FOLD2 = KB == 2 && VB == 2 && !VGROUP && QSPLIT;
    // bf16 with folded scales: the codes of channel d enter the MMA as
    // F_d * c + H_d (int2_biased(): the magic-exponent value, no subtraction,
    // F_d a power of 4) and both are removed exactly: K: the query channel is
    // pre-multiplied by 1 / F_d and scores start from -sum_d q'_d H_d / F_d;
    // V: at each flush O_d = (O_d - H_d sum_t p'_t) / F_d, the sum taken over
    // the same rounded P' the MMA consumes.
    constexpr bool FOLD2B = FOLD2 && DT == FADE_BF16;
    // bf16 with folded 2-bit scales: the QK product runs in fp16 with one
    // query part.  The fp32 query q'_d = q_rot,d * s_d / F_d is rounded once
    // to fp16 (11 significant bits, more than the hi + lo split in bf16 would
    // need MMAs for), after scaling each query row by a power of two 2^-e_r
    // that brings its largest |q'| into [2^13, 2^14) (no fp16 overflow,
    // normal values); the softmax applies 2^e_r with the score scale.  The
    // K codes enter as fp16(1024 + F_d * (code + 2)) (1 shift per 16 codes).
    // The PV product stays in bf16.
    constexpr bool QK16 = FOLD2B;
    constexpr int QDT = QK16 ? FADE_F16 : DT;
    using PQ = Pk<QDT>;
    constexpr int NQ = (QSPLIT && !QK16) ? 2 : 1;
    // QK accumulators split in two (shorter dependent MMA chains) where the
    // registers allow it without spilling
    constexpr bool kSplitAcc = KB == 2 || (!QSPLIT && !VGROUP);

    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base, derived from smem_raw by pointer arithmetic (not
    // an integer round trip) so every pointer taken from it stays in the
    // shared address space and its loads compile to shared, not generic, loads
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    constexpr int G = L::G, NS = L::NS;
    constexpr int PRODUCER = G * kConsumerWarps;   // first producer warp (one per group)
    constexpr int FPWARP = PRODUCER + G;            // the FP-tier warp
    const uint32_t bar_base = smem_u32(smem + L::BAR_OFF);
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (NS + s); };

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const bool is_producer = warp >= PRODUCER && warp < FPWARP;
    const int Z = p.B * p.Hkv;
    const int U = total_units(p, Z);
    // Never more CTAs than units, so every working CTA owns at least one unit
    // (the merge counts arrivals per row by CTA range).
    // Streaming CTAs: never more than units, so each owns at least one unit.
    // Every launched CTA runs the FP warp (rows split over the whole grid).
    const int C = p.n_ctas < U ? p.n_ctas : U;
    const int c = blockIdx.x;
    const bool streams = c < C;
    const int ub = streams ? (int)((int64_t)c * U / C) : 0;
    const int ue = streams ? (int)((int64_t)(c + 1) * U / C) : 0;

    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::FLAG_OFF);
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < NS; ++s) {
            mbar_init(full_bar(s), 32);
            mbar_init(empty_bar(s), kConsumerWarps * 32);   // every consumer lane arrives
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    // Inputs may be produced by the previous kernel in the stream (age-out,
    // query rotation): wait for it before touching global memory, then let the
    // next kernel in the stream start its prologue.  With `early` the tiers
    // are known not to be written by that kernel: the producer starts
    // streaming at once and only the consumers (queries, partial slots) wait.
    // The FP warp, too, streams its cache tiers before the dependency with
    // `early`; it waits itself before touching q, the new token or the workspace.
    const bool fp_early = p.early && warp == FPWARP;
    if (!(p.early && is_producer) && !fp_early) griddep_wait();
    if (warp < PRODUCER) griddep_launch_dependents();
    if (warp == FPWARP) {
        fp_rows_warp<DT, D, NT>(p, c, (int)gridDim.x, smem + L::AB_OFF, !fp_early);
        return;
    }
    if (ub >= ue) return;

    if (is_producer) {
        // ------------------------------ producers ------------------------------
        // One warp per consumer group, each filling only its group's slots
        // (stages g, g+G, ...), so a group that pauses (row flush) never
        // holds back the other groups' stages.
        const int pg = warp - PRODUCER;
        const uint64_t policy = evict_first_policy();
        if (lane == 0) {
            prefetch_tmap(&tmap_k);
            prefetch_tmap(&tmap_v);
            if (p.scale_tma) prefetch_tmap(&tmap_s);
        }
        int z = z_of_unit(p, Z, ub);
        int zb = units_begin(p, z), ze = units_begin(p, z + 1);
        // per-row values refreshed only when the row changes
        int64_t zrow0 = seg_row0(p, z), zlen = seg_len(p, z / p.Hkv);
        int s = pg;            // ring slot of stage i (i % NS), and its phase parity
        uint32_t ph = 0;
        for (int i = pg; ub + i < ue; i += G, s += G) {
            if (s >= NS) { s -= NS; ph ^= 1u; }
            const int u = ub + i;
            if (u >= ze) {
                while (u >= ze) { ++z; zb = ze; ze = units_begin(p, z + 1); }
                zrow0 = seg_row0(p, z);
                zlen = seg_len(p, z / p.Hkv);
            }
            if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.ws_err)) continue;
            const int64_t tok0 = (int64_t)(u - zb) * kStageTokens;
            // a unit is one page of a paged middle (kStageTokens == FADE_PAGE_TOKENS)
            const int64_t row0 = p.page_table
                ? (int64_t)__ldg(p.page_table + (int64_t)z * p.pages_per_row + (u - zb)) * kStageTokens
                : zrow0 + tok0;
            const int64_t len = zlen;
            uint8_t* st = smem + s * L::STAGE_BYTES;
            // Units past this row's length (uniform grid over a capacity bound)
            // carry no tokens: complete the stage without a copy.
            uint8_t* scs = smem + L::SC_BASE + s * L::SC_BYTES;
            if (lane == 0 && tok0 < len) {
                const uint32_t sc_bytes = p.scale_tma ? (uint32_t)L::sc_box_bytes(p.group) : 0u;
                mbar_expect_tx(full_bar(s), (uint32_t)(L::K_BYTES + L::V_BYTES) + sc_bytes);
                // maps address 128-byte rows: token row0 starts at row0*RB/128
                tma_load_2d(smem_u32(st + L::K_OFF), &tmap_k, 0, (int)(row0 * L::RBK / 128), full_bar(s), policy);
                tma_load_2d(smem_u32(st + L::V_OFF), &tmap_v, 0, (int)(row0 * L::RBV / 128), full_bar(s), policy);
                if (p.scale_tma) {
                    // per-token: 1-D map over rows; grouped: 2-D map [groups][D].
                    // Past the map's extent the TMA unit writes zeros.
                    if constexpr (!VGROUP) tma_load_1d(smem_u32(scs), &tmap_s, (int)row0, full_bar(s), policy);
                    else tma_load_2d(smem_u32(scs), &tmap_s, 0, (int)(row0 / p.group), full_bar(s), policy);
                }
            }
            if (!p.scale_tma && tok0 < len) {
                uint16_t* sc = reinterpret_cast<uint16_t*>(scs);
                if constexpr (!VGROUP) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int tt = lane * 4 + j;
                        sc[tt] = (tok0 + tt < len) ? load_bits<DT>(p.v_scale, row0 + tt) : (uint16_t)0;
                    }
                } else {
                    const int G = p.group;
                    const int ngr = kStageTokens / G;
                    const int64_t g0 = row0 / G;
                    for (int e = lane; e < ngr * D; e += 32) {
                        const int gi = e / D, d = e % D;
                        sc[e] = (tok0 + (int64_t)gi * G < len) ? load_bits<DT>(p.v_scale, (g0 + gi) * D + d)
                                                                : (uint16_t)0;
                    }
                }
            }
            mbar_arrive(full_bar(s));
        }
        // Drain: wait until the group released every stage still in flight,
        // so no TMA write targets this CTA's shared memory after it exits:
        // the waits the group's next NS/G stages would make.
        const int n = ue - ub;
        int i_next = pg;
        while (i_next < n) i_next += G;
        for (int k = 0; k < NS / G; ++k) {
            const int i = i_next + k * G;
            if (i - NS < 0) continue;   // that slot was never used
            const int s = i % NS;
            const uint32_t ph = (uint32_t)(i / NS) & 1u;
            mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.ws_err);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    const int grp = warp / kConsumerWarps;   // consumer group
    const int gw = warp % kConsumerWarps;    // warp within the group
    const int gid = lane >> 2, t = lane & 3;
    const int ctid = gw * 32 + lane;         // 0..127 within the group
    const int bar_id = 1 + grp;              // the group's named barrier
    const TileOffs<L::NCHK> koffs(gw * 32, lane);
    const TileOffs<L::NCHV> voffs(gw * 32, lane);
    float* mlbuf = reinterpret_cast<float*>(smem + L::RING_BYTES + grp * L::ML_BYTES);
    uint32_t qf[NQ][NT][KSTEPS][2];  // B fragments (exact model-dtype query)
    uint32_t ksc[KSTEPS][2];         // K scale pairs matching the A pairs
    float m_run[NT][2], l_run[NT][2];
    float kb[NT][2];                 // FOLD2B: 130 * sum of the row's query channels
    float qsr[NT][2];                // QK16: score scale of the C-fragment columns (qk_scale * 2^e_r)
    float lp[NT][2];                 // FOLD2B: running sum of the rounded P' of the row
    float o[NT][MT][4];
    int cur_z = -1, z_first = 0;
    int64_t cur_len = 0;

    // Each thread's K channels form, per 16-byte chunk cb of a packed row, one
    // contiguous block of CH channels starting at cb*CHW + CH*t; q and the K
    // scales are fetched block-wise (16-byte loads when aligned) and placed in
    // the fragment order given by KMap::kdim.
    constexpr int CH = (KB == 4) ? 8 : 16;
    constexpr int CHW = 4 * CH;
    auto load_block_bits = [&](const void* base, int64_t off, uint16_t (&e)[CH]) {
        const uint16_t* ptr = reinterpret_cast<const uint16_t*>(base) + off;
        if (p.q_vec) {
#pragma unroll
            for (int c4 = 0; c4 < CH / 8; ++c4) {
                const uint4 raw = __ldg(reinterpret_cast<const uint4*>(ptr) + c4);
                const uint16_t* r16 = reinterpret_cast<const uint16_t*>(&raw);
#pragma unroll
                for (int j = 0; j < 8; ++j) e[c4 * 8 + j] = r16[j];
            }
        } else {
#pragma unroll
            for (int j = 0; j < CH; ++j) e[j] = ptr[j];
        }
    };
    auto setup_z = [&](int z) {
        const int b = z / p.Hkv, h = z % p.Hkv;
        const int64_t ks_off = (int64_t)b * p.ks_sb + (int64_t)h * p.ks_sh;
#pragma unroll
        for (int cb = 0; cb < KSTEPS * 16 / CHW; ++cb) {
            uint16_t e[CH];
            load_block_bits(p.k_scale, ks_off + cb * CHW + CH * t, e);
#pragma unroll
            for (int u = 0; u < CHW / 16; ++u) {
                const int ks = cb * (CHW / 16) + u;
#pragma unroll
                for (int hs = 0; hs < 2; ++hs) {
                    const int i0 = KMap::kdim(ks, 2 * hs, t) - cb * CHW - CH * t;
                    const int i1 = KMap::kdim(ks, 2 * hs + 1, t) - cb * CHW - CH * t;
                    ksc[ks][hs] = (uint32_t)e[i0] | ((uint32_t)e[i1] << 16);
                }
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int r = nt * 8 + gid;
            const bool rv = r < p.rows;
            const int j = rv ? r / p.n_q : 0, sq = rv ? r % p.n_q : 0;
            const int64_t qoff = (int64_t)b * p.q_sb + (int64_t)(h * p.g + j) * p.q_sh + (int64_t)sq * p.q_ss;
            // fp32 query chunk cb of this lane's row (rotated tiers), with the
            // K scales folded in (FOLD2)
            auto load_qrow = [&](int cb, float (&e)[CH]) {
                const float* ptr = reinterpret_cast<const float*>(p.q) + qoff + cb * CHW + CH * t;
#pragma unroll
                for (int c4 = 0; c4 < CH / 4; ++c4) {
                    const float4 v4 = rv ? __ldg(reinterpret_cast<const float4*>(ptr) + c4)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
                    e[4 * c4] = v4.x; e[4 * c4 + 1] = v4.y; e[4 * c4 + 2] = v4.z; e[4 * c4 + 3] = v4.w;
                }
                if constexpr (FOLD2) {
                    uint16_t kse[CH];
                    load_block_bits(p.k_scale, ks_off + cb * CHW + CH * t, kse);
#pragma unroll
                    for (int jj = 0; jj < CH; ++jj) e[jj] *= P::unpack_lo((uint32_t)kse[jj]);
                }
            };
            // QK16: the row's power-of-two normalisation 2^-sh (lanes 4 gid ..
            // 4 gid + 3 hold the row's channels)
            float rsc = 1.f;
            if constexpr (QK16) {
                float amax = 0.f;
#pragma unroll
                for (int cb = 0; cb < KSTEPS * 16 / CHW; ++cb) {
                    float e[CH];
                    load_qrow(cb, e);
#pragma unroll
                    for (int jj = 0; jj < CH; ++jj) {
                        const int d = cb * CHW + CH * t + jj;
                        amax = fmaxf(amax, fabsf(e[jj] * kInvF2h(d)));
                    }
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                int ex = 0;
                if (amax > 0.f && amax < INFINITY) frexpf(amax, &ex);
                const int sh = (amax > 0.f && amax < INFINITY) ? ex - 14 : 0;
                rsc = ldexpf(1.f, -sh);
                const float rq = ldexpf(p.qk_scale, sh);
                qsr[nt][0] = __shfl_sync(0xffffffffu, rq, (2 * t) * 4);
                qsr[nt][1] = __shfl_sync(0xffffffffu, rq, (2 * t + 1) * 4);
            } else {
                qsr[nt][0] = qsr[nt][1] = p.qk_scale;
            }
#pragma unroll
            for (int cb = 0; cb < KSTEPS * 16 / CHW; ++cb) {
                if constexpr (QSPLIT) {
                    float e[CH];
                    load_qrow(cb, e);
#pragma unroll
                    for (int u = 0; u < CHW / 16; ++u) {
                        const int ks = cb * (CHW / 16) + u;
#pragma unroll
                        for (int hs = 0; hs < 2; ++hs) {
                            const int d0 = KMap::kdim(ks, 2 * hs, t), d1 = KMap::kdim(ks, 2 * hs + 1, t);
                            float v0 = e[d0 - cb * CHW - CH * t];
                            float v1 = e[d1 - cb * CHW - CH * t];
                            if constexpr (QK16) {   // powers of 2: exact
                                v0 *= kInvF2h(d0) * rsc;
                                v1 *= kInvF2h(d1) * rsc;
                            } else if constexpr (FOLD2B) {
                                v0 *= kInvF2(d0);
                                v1 *= kInvF2(d1);
                            }
                            const uint32_t hp = PQ::pack(v0, v1);
                            qf[0][nt][ks][hs] = hp;
                            if constexpr (NQ == 2) {
                                const float h0 = PQ::unpack_lo(hp), h1 = PQ::unpack_lo(hp >> 16);
                                qf[1][nt][ks][hs] = PQ::pack(v0 - h0, v1 - h1);
                            }
                        }
                    }
                } else {
                    uint16_t e[CH];
                    if (rv) load_block_bits(p.q, qoff + cb * CHW + CH * t, e);
                    else {
#pragma unroll
                        for (int jj = 0; jj < CH; ++jj) e[jj] = 0;
                    }
#pragma unroll
                    for (int u = 0; u < CHW / 16; ++u) {
                        const int ks = cb * (CHW / 16) + u;
#pragma unroll
                        for (int hs = 0; hs < 2; ++hs) {
                            const int i0 = KMap::kdim(ks, 2 * hs, t) - cb * CHW - CH * t;
                            const int i1 = KMap::kdim(ks, 2 * hs + 1, t) - cb * CHW - CH * t;
                            qf[0][nt][ks][hs] = (uint32_t)e[i0] | ((uint32_t)e[i1] << 16);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m_run[nt][0] = m_run[nt][1] = kMaskedMax;
            l_run[nt][0] = l_run[nt][1] = 0.f;
            lp[nt][0] = lp[nt][1] = 0.f;
#pragma unroll
            for (int mi = 0; mi < MT; ++mi)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[nt][mi][e] = 0.f;
            if constexpr (FOLD2B) {
                // this lane's query channels (row gid), both hi and lo parts
                float sum = 0.f;
#pragma unroll
                for (int qs = 0; qs < NQ; ++qs)
#pragma unroll
                    for (int ks = 0; ks < KSTEPS; ++ks)
#pragma unroll
                        for (int hs = 0; hs < 2; ++hs)
                            if constexpr (QK16)
                                sum += kH2h(KMap::kdim(ks, 2 * hs, t)) * PQ::unpack_lo(qf[qs][nt][ks][hs]) +
                                       kH2h(KMap::kdim(ks, 2 * hs + 1, t)) * PQ::unpack_lo(qf[qs][nt][ks][hs] >> 16);
                            else
                                sum += kH2(KMap::kdim(ks, 2 * hs, t)) * P::unpack_lo(qf[qs][nt][ks][hs]) +
                                       kH2(KMap::kdim(ks, 2 * hs + 1, t)) * P::unpack_lo(qf[qs][nt][ks][hs] >> 16);
                sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                // C-fragment columns 2t, 2t+1 are query rows held by lanes 8t, 8t+4
                kb[nt][0] = __shfl_sync(0xffffffffu, sum, (2 * t) * 4);
                kb[nt][1] = __shfl_sync(0xffffffffu, sum, (2 * t + 1) * 4);
            }
        }
        cur_len = seg_len(p, b);
    };

    // Row boundary: combine the 4 consumer warps' online-softmax states into
    // one CTA partial and store it at the row's slot for this CTA (the first
    // unit of the row it processed).  Plain stores only: the finisher kernel
    // reads the partials after this grid has completed, so no fence, counter
    // or merge sits on the streaming path.  The warps are summed in a fixed
    // order ((w0 + w2) + (w1 + w3)): repeated calls give identical bits.
    constexpr int MLW = NT * 8;   // rows per gw in the statistics buffer
    int n_flush = 0;
    auto flush = [&](int z, float* scratch) {
        // 1) complete the per-thread row sums over the 8 token lanes
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                float l = l_run[nt][e];
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                l_run[nt][e] = l;
            }
        // statistics alternate between two buffers: a gw can reach the next
        // flush while threads 0..rows-1 still read this one's
        float* mlw = mlbuf + (n_flush & 1) * (kConsumerWarps * MLW * 2);
        ++n_flush;
        if (gid == 0) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int r = nt * 8 + 2 * t + e;
                    mlw[(gw * MLW + r) * 2 + 0] = m_run[nt][e];
                    mlw[(gw * MLW + r) * 2 + 1] = l_run[nt][e];
                }
        }
        named_bar_sync(bar_id, kConsumerWarps * 32);
        if constexpr (FOLD2B) {   // remove the code bias and factor: O_d = (O_d - H_d sum_t P') / F_d
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float q = lp[nt][e];
                    q += __shfl_xor_sync(0xffffffffu, q, 4);
                    q += __shfl_xor_sync(0xffffffffu, q, 8);
                    q += __shfl_xor_sync(0xffffffffu, q, 16);
#pragma unroll
                    for (int mi = 0; mi < MT; ++mi) {
                        // C-fragment rows gid, gid + 8 are channels vdim(mi, 0 / 1, gid); d % 4 = 2 (mi % 2) + hr
                        const int d0 = 2 * (mi & 1), d1 = 2 * (mi & 1) + 1;
                        o[nt][mi][e] = (o[nt][mi][e] - kH2(d0) * q) * kInvF2(d0);
                        o[nt][mi][e + 2] = (o[nt][mi][e + 2] - kH2(d1) * q) * kInvF2(d1);
                    }
                }
        }
        // 2) rescale this gw's O to the CTA max
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int r = nt * 8 + 2 * t + e;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mlw[(w * MLW + r) * 2]);
                const float f = (m_run[nt][e] == -INFINITY) ? 0.f : ex2(m_run[nt][e] - M);
#pragma unroll
                for (int mi = 0; mi < MT; ++mi) {
                    o[nt][mi][e] *= f;
                    o[nt][mi][e + 2] *= f;
                }
            }
        // 3) combine the 4 warps in the scratch buffer (the group's stage that
        //    was just consumed): FR regions of one warp's [rows][D] each; warps
        //    0..FR-1 store, the others add in turn, always in the same order
        //    (deterministic).  Channel pairs d, d+1 are adjacent: float2 stores.
        constexpr int WB = NT * 8 * D * 4;                                  // one warp's partial
        constexpr int FR = (L::STAGE_BYTES / WB) >= 4 ? 4 : ((L::STAGE_BYTES / WB) >= 2 ? 2 : 1);
        static_assert(L::STAGE_BYTES >= WB, "stage buffer too small for a partial");
        float* region = scratch + (gw % FR) * (NT * 8 * D);
        for (int pass = 0; pass < kConsumerWarps / FR; ++pass) {
            if (gw / FR == pass) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int r = nt * 8 + 2 * t + e;
                        if (r >= p.rows) continue;
#pragma unroll
                        for (int mi = 0; mi < MT; ++mi) {
                            float2* dst = reinterpret_cast<float2*>(region + r * D + VMap::vdim(mi, 0, gid));
                            float2 v = make_float2(o[nt][mi][e], o[nt][mi][e + 2]);
                            if (pass > 0) {
                                const float2 a2 = *dst;
                                v.x += a2.x;
                                v.y += a2.y;
                            }
                            *dst = v;
                        }
                    }
            }
            named_bar_sync(bar_id, kConsumerWarps * 32);
        }
        // 4) store the partial (float4 rows) at the first unit of z this
        //    group processed (unique per group and row)
        const int slot = z_first;
        float4* go = reinterpret_cast<float4*>(p.ws_o + (int64_t)slot * p.rows * D);
        for (int i = ctid; i < p.rows * D / 4; i += kConsumerWarps * 32) {
            float4 acc = reinterpret_cast<const float4*>(scratch)[i];
#pragma unroll
            for (int rg = 1; rg < FR; ++rg) {
                const float4 x = reinterpret_cast<const float4*>(scratch + rg * (NT * 8 * D))[i];
                acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
            }
            go[i] = acc;
        }
        if (ctid < p.rows) {
            const int r = ctid;
            float M = -INFINITY, Ls = 0.f;
            for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mlw[(w * MLW + r) * 2]);
            for (int w = 0; w < kConsumerWarps; ++w) {
                const float mw = mlw[(w * MLW + r) * 2];
                if (mw != -INFINITY) Ls += ex2(mw - M) * mlw[(w * MLW + r) * 2 + 1];
            }
            *reinterpret_cast<float2*>(p.ws_ml + ((int64_t)slot * p.rows + r) * 2) = make_float2(M, Ls);
        }
    };

    int z = z_of_unit(p, Z, ub);
    int zb = units_begin(p, z), ze = units_begin(p, z + 1);

    int s = grp;            // ring slot of stage i = i % NS
    uint32_t ph = 0;        // its phase parity = (i / NS) & 1
    for (int i = grp; ub + i < ue; i += G) {
        const int u = ub + i;
        while (u >= ze) { ++z; zb = ze; ze = units_begin(p, z + 1); }
        if (z != cur_z) {
            setup_z(z);
            cur_z = z;
            z_first = u;
        }
        const bool ready = mbar_wait(full_bar(s), ph, abort_flag, p.ws_err);
        const int tw = (u - zb) * kStageTokens + gw * 32;  // first token of this gw (row-relative)
        const int clen = (int)cur_len;
        const uint8_t* st = smem + s * L::STAGE_BYTES;
        const uint32_t kbase = smem_u32(st + L::K_OFF);
        const uint32_t vbase = smem_u32(st + L::V_OFF);
        const uint8_t* scb = smem + L::SC_BASE + s * L::SC_BYTES;

        if (ready && tw < clen) {
            // ---- S^T = K_deq . q^T for the gw's 2 m-tiles ----
            float sacc[2][NT][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) sacc[mt][nt][e] = FOLD2B ? -kb[nt][e & 1] : 0.f;
                // Two accumulators per tile halve the dependent MMA chain: the
                // low query part (or the odd k-steps) goes to sacc2.
                float sacc2[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) sacc2[nt][e] = 0.f;
                auto acc = [&](int ks, int qs, int nt) -> float (&)[4] {
                    return kSplitAcc && (NQ == 2 ? qs == 1 : (ks & 1) == 1) ? sacc2[nt] : sacc[mt][nt];
                };
                uint32_t kr[2][L::NCHK];
                load_tiles_at<L::NCHK, false>(kbase, koffs, mt, kr);
#pragma unroll
                for (int cb = 0; cb < L::NCHK; ++cb) {
                    if constexpr (KB == 4) {
                        uint32_t h0[4], h1[4];
                        Conv<DT>::int4(kr[0][cb], h0);
                        Conv<DT>::int4(kr[1][cb], h1);
#pragma unroll
                        for (int u2 = 0; u2 < 2; ++u2) {
                            const int ks = cb * 2 + u2;
                            const uint32_t a0 = P::mul(h0[2 * u2], ksc[ks][0]);
                            const uint32_t a1 = P::mul(h1[2 * u2], ksc[ks][0]);
                            const uint32_t a2 = P::mul(h0[2 * u2 + 1], ksc[ks][1]);
                            const uint32_t a3 = P::mul(h1[2 * u2 + 1], ksc[ks][1]);
#pragma unroll
                            for (int qs = 0; qs < NQ; ++qs)
#pragma unroll
                                for (int nt = 0; nt < NT; ++nt)
                                    PQ::mma(acc(ks, qs, nt), a0, a1, a2, a3,
                                            qf[qs][nt][ks][0], qf[qs][nt][ks][1]);
                        }
                    } else {
                        uint32_t h0[8], h1[8];
                        if constexpr (FOLD2B) {
                            Conv<QDT>::int2_biased(kr[0][cb], h0);
                            Conv<QDT>::int2_biased(kr[1][cb], h1);
                        } else {
                            Conv<DT>::int2(kr[0][cb], h0);
                            Conv<DT>::int2(kr[1][cb], h1);
                        }
#pragma unroll
                        for (int u4 = 0; u4 < 4; ++u4) {
                            const int ks = cb * 4 + u4;
                            const uint32_t a0 = FOLD2 ? h0[2 * u4] : P::mul(h0[2 * u4], ksc[ks][0]);
                            const uint32_t a1 = FOLD2 ? h1[2 * u4] : P::mul(h1[2 * u4], ksc[ks][0]);
                            const uint32_t a2 = FOLD2 ? h0[2 * u4 + 1] : P::mul(h0[2 * u4 + 1], ksc[ks][1]);
                            const uint32_t a3 = FOLD2 ? h1[2 * u4 + 1] : P::mul(h1[2 * u4 + 1], ksc[ks][1]);
#pragma unroll
                            for (int qs = 0; qs < NQ; ++qs)
#pragma unroll
                                for (int nt = 0; nt < NT; ++nt)
                                    PQ::mma(acc(ks, qs, nt), a0, a1, a2, a3,
                                            qf[qs][nt][ks][0], qf[qs][nt][ks][1]);
                        }
                    }
                }
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) sacc[mt][nt][e] += sacc2[nt][e];
            }
            // ---- online softmax over the 32 tokens (log2 domain) ----
            // Scores stay unscaled; the running maxima are in scaled units
            // (qk_scale > 0 keeps the order) and exp2(s * qk_scale - m) is one
            // FMA.  Running maxima start at kMaskedMax (finite), so masked
            // scores (-inf) give exp2 = 0 and no difference of infinities arises.
            const float qks = p.qk_scale;
            if (tw + 32 > clen) {   // gw-uniform: only the row's last tile is partial
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            if (tw + mt * 16 + gid + ((e >> 1) << 3) >= clen) sacc[mt][nt][e] = -INFINITY;
            }
            uint32_t pb[2][NT][2];
            {
            // Lazy maxima: while every score of the stage stays within 2^8 of
            // its row's running maximum (log2 units), the maxima are kept and
            // the weights (<= 256, finite in the model dtype) use them as is;
            // the shuffle reduction and rescale run only when some row exceeds
            // that margin.  Maxima start at kMaskedMax, so a row's first stage
            // always takes the full path.
            bool full = true;
            {
                bool need = false;
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float lm = fmaxf(fmaxf(sacc[0][nt][e], sacc[0][nt][e + 2]),
                                               fmaxf(sacc[1][nt][e], sacc[1][nt][e + 2]));
                        need |= lm * (QK16 ? qsr[nt][e] : qks) > m_run[nt][e] + 8.f;
                    }
                full = __any_sync(0xffffffffu, need);
            }
            if (full) {
            bool grow = false;
            float corr[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    float mx = fmaxf(fmaxf(sacc[0][nt][e], sacc[0][nt][e + 2]),
                                     fmaxf(sacc[1][nt][e], sacc[1][nt][e + 2]));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    const float mnew = fmaxf(m_run[nt][e], mx * (QK16 ? qsr[nt][e] : qks));
                    grow |= mnew > m_run[nt][e];
                    corr[nt][e] = ex2(m_run[nt][e] - mnew);
                    m_run[nt][e] = mnew;
                }
            }
            // Rescale only when some row maximum of the gw grew (corr is
            // exactly 1 otherwise, so skipping is bit-identical).
            if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        l_run[nt][e] *= corr[nt][e];
                        lp[nt][e] *= corr[nt][e];
#pragma unroll
                        for (int mi = 0; mi < MT; ++mi) {
                            o[nt][mi][e] *= corr[nt][e];
                            o[nt][mi][e + 2] *= corr[nt][e];
                        }
                    }
            }
            }   // full
            // FOLD2: V scales of the C-fragment rows (tokens gid, gid + 8 of
            // each m-tile); zero past the length, where the bytes are stale
            float tsc[2][2];
            if constexpr (FOLD2) {
                const uint16_t* sc16 = reinterpret_cast<const uint16_t*>(scb);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int hr = 0; hr < 2; ++hr) {
                        const int tl = gw * 32 + mt * 16 + gid + 8 * hr;
                        tsc[mt][hr] = (tw - gw * 32 + tl < clen) ? P::unpack_lo((uint32_t)sc16[tl]) : 0.f;
                    }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    float pv[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float pe = ex2(fmaf(sacc[mt][nt][e], QK16 ? qsr[nt][e & 1] : qks, -m_run[nt][e & 1]));
                        l_run[nt][e & 1] += pe;
                        pv[e] = FOLD2 ? pe * tsc[mt][e >> 1] : pe;
                    }
                    const uint32_t p01 = P::pack(pv[0], pv[1]), p23 = P::pack(pv[2], pv[3]);
                    if constexpr (FOLD2B) {   // exactly the P' the MMA sees
                        lp[nt][0] += P::unpack_lo(p01) + P::unpack_lo(p23);
                        lp[nt][1] += P::unpack_lo(p01 >> 16) + P::unpack_lo(p23 >> 16);
                    }
                    pb[mt][nt][0] = movmatrix_t(p01);
                    pb[mt][nt][1] = movmatrix_t(p23);
                }
            }
            }   // softmax
            // ---- O^T += V_deq^T . P^T ----
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const int trow0 = gw * 32 + mt * 16;
                uint32_t vr[2][L::NCHV];
                load_tiles_at<L::NCHV, true>(vbase, voffs, mt, vr);
                // tokens of this m-tile past the length: their scales may be
                // stale bytes (NaN * 0 must not reach the MMA), so zero them;
                // a tile entirely past the length is skipped.
                const int tile_tok = tw - gw * 32 + trow0;
                if (tile_tok >= clen) continue;
                uint32_t vs0 = 0, vs1 = 0;
                const uint16_t* gsc = nullptr;
                if constexpr (!VGROUP) {
                    const uint32_t* sc32 = reinterpret_cast<const uint32_t*>(scb);
                    vs0 = sc32[(trow0 + 2 * t) >> 1];       // tokens 2t, 2t+1
                    vs1 = sc32[(trow0 + 8 + 2 * t) >> 1];   // tokens 8+2t, 9+2t
                    const int rem = clen - tile_tok;  // valid tokens in this tile (> 0)
                    if (rem < 16) {
                        const int t0 = 2 * t, t1 = 8 + 2 * t;
                        vs0 &= (t0 < rem ? 0x0000FFFFu : 0u) | (t0 + 1 < rem ? 0xFFFF0000u : 0u);
                        vs1 &= (t1 < rem ? 0x0000FFFFu : 0u) | (t1 + 1 < rem ? 0xFFFF0000u : 0u);
                    }
                } else {
                    gsc = reinterpret_cast<const uint16_t*>(scb) + (trow0 / p.group) * D;
                }
#pragma unroll
                for (int cb = 0; cb < L::NCHV; ++cb) {
                    if constexpr (VB == 4) {
                        uint32_t h0[4], h1[4];
                        Conv<DT>::int4(vr[0][cb], h0);   // tokens 2t,2t+1
                        Conv<DT>::int4(vr[1][cb], h1);   // tokens 8+2t, 9+2t
                        // m-tile j: rows (gid: e_{2j} -> h[2j+1]), (gid+8: e_{2j+1} -> h[2j])
#pragma unroll
                        for (int j = 0; j < 2; ++j) {
                            const int mi = cb * 2 + j;
                            uint32_t a0, a1, a2, a3;
                            if constexpr (!VGROUP) {
                                a0 = P::mul(h0[2 * j + 1], vs0);
                                a1 = P::mul(h0[2 * j], vs0);
                                a2 = P::mul(h1[2 * j + 1], vs1);
                                a3 = P::mul(h1[2 * j], vs1);
                            } else {
                                const uint32_t g0 = dup16(gsc[VMap::vdim(mi, 0, gid)]);
                                const uint32_t g1 = dup16(gsc[VMap::vdim(mi, 1, gid)]);
                                a0 = P::mul(h0[2 * j + 1], g0);
                                a1 = P::mul(h0[2 * j], g1);
                                a2 = P::mul(h1[2 * j + 1], g0);
                                a3 = P::mul(h1[2 * j], g1);
                            }
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt)
                                P::mma(o[nt][mi], a0, a1, a2, a3, pb[mt][nt][0], pb[mt][nt][1]);
                        }
                    } else {
                        uint32_t h0[8], h1[8];
                        if constexpr (FOLD2B) {
                            Conv<DT>::int2_biased(vr[0][cb], h0);
                            Conv<DT>::int2_biased(vr[1][cb], h1);
                        } else {
                            Conv<DT>::int2(vr[0][cb], h0);
                            Conv<DT>::int2(vr[1][cb], h1);
                        }
                        // channels +0 h[3], +1 h[2], +2 h[1], +3 h[0], +4 h[7], +5 h[6], +6 h[5], +7 h[4]
                        const int lo[4] = {3, 1, 7, 5};
                        const int hi[4] = {2, 0, 6, 4};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int mi = cb * 4 + j;
                            uint32_t a0, a1, a2, a3;
                            if constexpr (FOLD2) {
                                a0 = h0[lo[j]];
                                a1 = h0[hi[j]];
                                a2 = h1[lo[j]];
                                a3 = h1[hi[j]];
                            } else if constexpr (!VGROUP) {
                                a0 = P::mul(h0[lo[j]], vs0);
                                a1 = P::mul(h0[hi[j]], vs0);
                                a2 = P::mul(h1[lo[j]], vs1);
                                a3 = P::mul(h1[hi[j]], vs1);
                            } else {
                                const uint32_t g0 = dup16(gsc[VMap::vdim(mi, 0, gid)]);
                                const uint32_t g1 = dup16(gsc[VMap::vdim(mi, 1, gid)]);
                                a0 = P::mul(h0[lo[j]], g0);
                                a1 = P::mul(h0[hi[j]], g1);
                                a2 = P::mul(h1[lo[j]], g0);
                                a3 = P::mul(h1[hi[j]], g1);
                            }
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt)
                                P::mma(o[nt][mi], a0, a1, a2, a3, pb[mt][nt][0], pb[mt][nt][1]);
                        }
                    }
                }
            }
        }
        // The group's last stage of this row: combine and store the row's
        // partial in this stage's buffer before releasing it.
        if (ub + i + G >= ue || ub + i + G >= ze) {
            flush(cur_z, reinterpret_cast<float*>(smem + s * L::STAGE_BYTES));
            // the buffer was written through the generic proxy; the next TMA
            // load into it is an async-proxy write
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        mbar_arrive(empty_bar(s));   // each lane after its own reads of the stage
        s += G;
        if (s >= NS) { s -= NS; ph ^= 1u; }
    }
}

#include "middle_tc.cuh"

// ---------------------------------------------------------------------------
// k0: q_rot = q @ R^T (fp32), kRotRows query rows per CTA
// ---------------------------------------------------------------------------
constexpr int kRotRows = 16;   // query rows per rotate_queries CTA
constexpr int kRotQS = 20;     // padded row of the transposed query tile (16-byte multiple)

// q_rot[row][d] = sum_e q[row][e] * R[d][e] in fp32 (FMA, e ascending:
// deterministic).  2 * D threads per CTA, each owning a 2-row x 4-channel
// tile of the CTA's kRotRows x D block, so one e step is an 8-byte and a
// 16-byte shared load (2 query values, 4 consecutive R^T values) and 8 FMAs.
// R^T and the transposed query tile are staged in shared memory once per CTA
// with every global load of a thread issued before its stores (trip counts
// are compile-time), so staging costs about one L2 round trip, not one per
// load; R^T stores go lane -> channel, conflict-free.
template <int DT, int D>
__global__ void __launch_bounds__(2 * D) rotate_queries_kernel(const void* q, int Hq, int n_q, int64_t q_sb,
                                                             int64_t q_sh, int64_t q_ss,
                                                             const float* __restrict__ R,
                                                             float* __restrict__ q_rot, int n_rows) {
    constexpr int NT = 2 * D, D4 = D / 4;
    constexpr int RP = D * D4 / NT;          // float4 pieces of R per thread
    constexpr int QP = kRotRows * D / NT;    // query elements per thread
    extern __shared__ __align__(16) float rsm[];
    float* rt = rsm;               // [D][D]: rt[e*D + d] = R[d][e]
    float* qt = rsm + D * D;       // [D][kRotQS]: qt[e*kRotQS + r] = q[row0 + r][e]
    griddep_wait();                // q and R may come from the preceding kernel
    griddep_launch_dependents();
    const int tid = threadIdx.x;
    const int row0 = blockIdx.x * kRotRows;
    const int nr = (n_rows - row0) < kRotRows ? (n_rows - row0) : kRotRows;
    float4 r4[RP];
    float qv[QP];
#pragma unroll
    for (int k = 0; k < RP; ++k) {
        const int i = tid + k * NT, d = i % D, e = (i / D) * 4;
        r4[k] = __ldg(reinterpret_cast<const float4*>(R + d * D + e));
    }
#pragma unroll
    for (int k = 0; k < QP; ++k) {
        const int i = tid + k * NT, r = i / D, e = i % D;
        qv[k] = 0.f;
        if (r < nr) {
            const int row = row0 + r;   // (b*Hq + hq)*n_q + s
            const int s = row % n_q, bh = row / n_q;
            const int hq = bh % Hq, b = bh / Hq;
            qv[k] = load_f<DT>(q, (int64_t)b * q_sb + (int64_t)hq * q_sh + (int64_t)s * q_ss + e);
        }
    }
#pragma unroll
    for (int k = 0; k < RP; ++k) {
        const int i = tid + k * NT, d = i % D, e = (i / D) * 4;
        rt[e * D + d] = r4[k].x;
        rt[(e + 1) * D + d] = r4[k].y;
        rt[(e + 2) * D + d] = r4[k].z;
        rt[(e + 3) * D + d] = r4[k].w;
    }
#pragma unroll
    for (int k = 0; k < QP; ++k) {
        const int i = tid + k * NT;
        qt[(i % D) * kRotQS + i / D] = qv[k];
    }
    __syncthreads();
    const int tc = tid % D4, tr = tid / D4;   // channels 4tc.., rows 2tr, 2tr+1
    float acc[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
#pragma unroll 8
    for (int e = 0; e < D; ++e) {
        const float2 qa = *reinterpret_cast<const float2*>(qt + e * kRotQS + 2 * tr);
        const float4 rv = *reinterpret_cast<const float4*>(rt + e * D + 4 * tc);
        const float ra[4] = {rv.x, rv.y, rv.z, rv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc[0][j] = fmaf(qa.x, ra[j], acc[0][j]);
            acc[1][j] = fmaf(qa.y, ra[j], acc[1][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int r = 2 * tr + i;
        if (r < nr)
            *reinterpret_cast<float4*>(q_rot + (int64_t)(row0 + r) * D + 4 * tc) =
                make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    }
}

// ---------------------------------------------------------------------------
// k2: finisher, one CTA per (b, kv-head).
//   Prologue (runs while the middle kernel's last CTAs drain; with no middle
//   it first waits for the previous kernel): attention over the FP tiers --
//   sinks and recent window -- from shared-memory chunks of up to kFinChunk
//   tokens gathered across the FP segments with 16-byte cp.async, giving an
//   un-normalised partial (m, l, O) in log2 units.
//   Then griddepcontrol.wait (the middle grid has completed and its partials
//   are visible), merge with every middle partial of the row (online over
//   chunks of kFinSlots partials), rotate the middle part back for rotated
//   tiers (out = fp + mid @ R), normalise and write `out`.
// ---------------------------------------------------------------------------
constexpr int kFinThreads = 256;
constexpr int kFinChunk = 128;   // FP tokens staged per pass
constexpr int kFinSlots = 64;    // middle partials merged per pass

struct FinParams {
    int B, Hq, Hkv, D, n_q, g, rows;
    float qk_scale;
    const void* q;
    int64_t q_sb, q_sh, q_ss;
    void* out;
    int64_t o_sb, o_sh, o_ss;
    int n_fp;
    FpSeg fp[FADE_MAX_SEGMENTS];
    int vec;                        // FP rows 16-byte aligned: cp.async staging
    int has_mid;                    // a middle kernel precedes this one
    const int32_t* cu_units;        // middle units per row (ragged) or null
    int units_per_z;
    int n_ctas;                     // middle grid (before clamping to the units)
    int groups;                     // consumer groups per middle CTA
    const float* ws_ml;             // middle partials [U][rows][2]
    const float* ws_o;              // [U][rows][D]
    const float* rotation;          // rotated middle: [D,D] fp32, else null
    // FP-tier partials and the fused age-out's new lengths (middle kernel)
    const float* ws_fpml;           // [Z][rows][2]
    const float* ws_fpo;            // [Z][rows][D]
    int age;
    int32_t* mid_len;
    const int* ws_age;              // [Z]
};

template <int D, int NT>
struct FinLayout {
    static constexpr int ROWS = NT * 8;
    static constexpr int KSTR = D + 8;                               // padded K row (elements)
    static constexpr int K_OFF = 0;                                  // [chunk][KSTR] dtype
    static constexpr int V_OFF = K_OFF + kFinChunk * KSTR * 2;       // [chunk][D] dtype
    static constexpr int Q_OFF = V_OFF + kFinChunk * D * 2;          // [ROWS][D] f32 (x qk_scale)
    static constexpr int P_OFF = Q_OFF + ROWS * D * 4;               // [ROWS][chunk] f32
    static constexpr int ST_OFF = P_OFF + ROWS * kFinChunk * 4;      // row stats [4][ROWS]
    static constexpr int SW_OFF = ST_OFF + 4 * ROWS * 4;             // [kFinSlots][ROWS] weights
    static constexpr int SL_OFF = SW_OFF + kFinSlots * ROWS * 4;     // [kFinSlots][ROWS] sums
    static constexpr int SLOT_OFF = SL_OFF + kFinSlots * ROWS * 4;   // [kFinSlots] partial slots
    static constexpr int BYTES = SLOT_OFF + kFinSlots * 4;
    static_assert(ROWS * D * 4 <= V_OFF, "rotation scratch reuses the K region");
};


template <int DT, int D, int NT>
__global__ void __launch_bounds__(kFinThreads)
finish_kernel(const __grid_constant__ FinParams p) {
    using L = FinLayout<D, NT>;
    using T = typename Elem<DT>::T;
    constexpr int ROWS = L::ROWS;
    constexpr int D2 = D / 2;
    constexpr int OUTS = (ROWS * D2 + kFinThreads - 1) / kFinThreads;   // (row, channel pair) per thread
    constexpr int NW = kFinThreads / 32;
    constexpr int PRE = 8;           // middle partials whose outputs are fetched with their statistics
    extern __shared__ __align__(16) uint8_t fsm[];
    T* ksm = reinterpret_cast<T*>(fsm + L::K_OFF);
    T* vsm = reinterpret_cast<T*>(fsm + L::V_OFF);
    float* qsm = reinterpret_cast<float*>(fsm + L::Q_OFF);
    float* psm = reinterpret_cast<float*>(fsm + L::P_OFF);
    float* m_row = reinterpret_cast<float*>(fsm + L::ST_OFF);
    float* l_row = m_row + ROWS;
    float* c_row = m_row + 2 * ROWS;   // per-pass rescale factor
    float* f_row = m_row + 3 * ROWS;   // 1 / L
    float* sw = reinterpret_cast<float*>(fsm + L::SW_OFF);
    float* sl = reinterpret_cast<float*>(fsm + L::SL_OFF);
    int* sslot = reinterpret_cast<int*>(fsm + L::SLOT_OFF);

    const int z = blockIdx.x;
    const int b = z / p.Hkv, h = z % p.Hkv;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    const int rows = p.rows;
    float acc_f[OUTS][2];
#pragma unroll
    for (int k = 0; k < OUTS; ++k) acc_f[k][0] = acc_f[k][1] = 0.f;

    float2 fp_ml = make_float2(-INFINITY, 0.f);   // FP-tier partial statistics of row tid
    if (p.has_mid) {
        // The middle kernel's FP warps computed the FP-tier partial of every
        // row (and the fused age-out): wait for that grid; the merge below
        // starts from that partial (its loads overlap the slot lookup).
        griddep_wait();
        griddep_launch_dependents();
        if (tid < rows) fp_ml = *reinterpret_cast<const float2*>(p.ws_fpml + ((int64_t)z * rows + tid) * 2);
#pragma unroll
        for (int k = 0; k < OUTS; ++k) {
            const int i = tid + k * kFinThreads;
            if (i < rows * D2) {
                const int r = i / D2, d2 = i % D2;
                const float2 v = *reinterpret_cast<const float2*>(p.ws_fpo + ((int64_t)z * rows + r) * D + 2 * d2);
                acc_f[k][0] = v.x;
                acc_f[k][1] = v.y;
            }
        }
        // the middle grid (every reader of the lengths) has completed: advance
        if (p.age && h == 0 && tid == 0) p.mid_len[b] = p.ws_age[z];
    } else {
        griddep_wait();
        griddep_launch_dependents();
        // ---- no quantised tier: attention over the FP segments here ----
        int64_t seg_len_[FADE_MAX_SEGMENTS], seg_row_[FADE_MAX_SEGMENTS];
        int64_t n_tok = 0;
#pragma unroll
        for (int s = 0; s < FADE_MAX_SEGMENTS; ++s) {
            seg_len_[s] = 0;
            seg_row_[s] = 0;
            if (s < p.n_fp) {
                const FpSeg& sg = p.fp[s];
                seg_len_[s] = sg.lens ? (int64_t)sg.lens[b] : sg.len;
                seg_row_[s] = sg.row_base ? sg.row_base[z] : (int64_t)b * sg.row_sb + (int64_t)h * sg.row_sh;
                n_tok += seg_len_[s];
            }
        }
        auto stage = [&](int64_t t0, int n) {
            constexpr int PCS = D / 8;   // 16-byte pieces per row
            for (int i = tid; i < n * PCS; i += kFinThreads) {
                const int tk = i / PCS, c = i % PCS;
                int64_t ft = t0 + tk;
                int s = 0;
                while (s < p.n_fp - 1 && ft >= seg_len_[s]) { ft -= seg_len_[s]; ++s; }
                const FpSeg& sg = p.fp[s];
                const int64_t off = (seg_row_[s] + ft) * D + c * 8;
                const T* ks = reinterpret_cast<const T*>(sg.k) + off;
                const T* vs = reinterpret_cast<const T*>(sg.v) + off;
                T* kd = ksm + tk * L::KSTR + c * 8;
                T* vd = vsm + tk * D + c * 8;
                if (p.vec) {
                    cp_async16(smem_u32(kd), ks);
                    cp_async16(smem_u32(vd), vs);
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        kd[e] = ks[e];
                        vd[e] = vs[e];
                    }
                }
            }
        };
        if (n_tok > 0) stage(0, (int)(n_tok < kFinChunk ? n_tok : kFinChunk));
        for (int i = tid; i < ROWS * D; i += kFinThreads) {
            const int r = i / D, d = i % D;
            float v = 0.f;
            if (r < rows) {
                const int j = r / p.n_q, sq = r % p.n_q;
                v = load_f<DT>(p.q, (int64_t)b * p.q_sb + (int64_t)(h * p.g + j) * p.q_sh + (int64_t)sq * p.q_ss + d) *
                    p.qk_scale;
            }
            qsm[i] = v;
        }
        if (tid < ROWS) { m_row[tid] = -INFINITY; l_row[tid] = 0.f; }
        for (int64_t t0 = 0; t0 < n_tok; t0 += kFinChunk) {
            const int n = (int)((n_tok - t0) < kFinChunk ? (n_tok - t0) : kFinChunk);
            if (t0 > 0) {
                __syncthreads();   // previous pass finished reading ksm / vsm / psm
                stage(t0, n);
            }
            cp_async_wait_all();
            __syncthreads();
            // ---- scores S[r][tok] = q_r . k_tok (log2 domain) ----
            for (int i = tid; i < rows * n; i += kFinThreads) {
                const int r = i / n, tk = i % n;
                const uint4* kr = reinterpret_cast<const uint4*>(ksm + tk * L::KSTR);
                const float4* qr = reinterpret_cast<const float4*>(qsm + r * D);
                float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
                for (int c = 0; c < D / 8; ++c) {
                    const uint4 raw = kr[c];
                    const T* e8 = reinterpret_cast<const T*>(&raw);
                    const float4 q0 = qr[2 * c], q1 = qr[2 * c + 1];
                    a0 = fmaf(q0.x, Elem<DT>::to_f(e8[0]), a0);
                    a1 = fmaf(q0.y, Elem<DT>::to_f(e8[1]), a1);
                    a0 = fmaf(q0.z, Elem<DT>::to_f(e8[2]), a0);
                    a1 = fmaf(q0.w, Elem<DT>::to_f(e8[3]), a1);
                    a0 = fmaf(q1.x, Elem<DT>::to_f(e8[4]), a0);
                    a1 = fmaf(q1.y, Elem<DT>::to_f(e8[5]), a1);
                    a0 = fmaf(q1.z, Elem<DT>::to_f(e8[6]), a0);
                    a1 = fmaf(q1.w, Elem<DT>::to_f(e8[7]), a1);
                }
                psm[r * kFinChunk + tk] = a0 + a1;
            }
            __syncthreads();
            // ---- online softmax per row (one warp per row) ----
            for (int r = warp; r < rows; r += NW) {
                float mx = -INFINITY;
                for (int tk = lane; tk < n; tk += 32) mx = fmaxf(mx, psm[r * kFinChunk + tk]);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                const float mold = m_row[r];
                const float mnew = fmaxf(mold, mx);
                float sum = 0.f;
                for (int tk = lane; tk < n; tk += 32) {
                    const float e = ex2(psm[r * kFinChunk + tk] - mnew);
                    psm[r * kFinChunk + tk] = e;
                    sum += e;
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                if (lane == 0) {
                    const float corr = (mold == -INFINITY) ? 0.f : ex2(mold - mnew);
                    m_row[r] = mnew;
                    l_row[r] = l_row[r] * corr + sum;
                    c_row[r] = corr;
                }
            }
            __syncthreads();
            // ---- O[r][d] = O * corr + sum_tok P[r][tok] V[tok][d] ----
#pragma unroll
            for (int k = 0; k < OUTS; ++k) {
                const int i = tid + k * kFinThreads;
                if (i >= rows * D2) continue;
                const int r = i / D2, d2 = i % D2;
                const float corr = c_row[r];
                float a0 = acc_f[k][0] * corr, a1 = acc_f[k][1] * corr;
                const float* pr = psm + r * kFinChunk;
                const uint32_t* vcol = reinterpret_cast<const uint32_t*>(vsm) + d2;
#pragma unroll 4
                for (int tk = 0; tk < n; ++tk) {
                    const uint32_t vv = vcol[tk * D2];
                    const float pt = pr[tk];
                    a0 = fmaf(pt, Elem<DT>::to_f(reinterpret_cast<const T*>(&vv)[0]), a0);
                    a1 = fmaf(pt, Elem<DT>::to_f(reinterpret_cast<const T*>(&vv)[1]), a1);
                }
                acc_f[k][0] = a0;
                acc_f[k][1] = a1;
            }
        }
    }

    // ---- merge the middle partials ----
    float acc_m[OUTS][2];
#pragma unroll
    for (int k = 0; k < OUTS; ++k) acc_m[k][0] = acc_m[k][1] = 0.f;
    int zb = 0, ze = 0, c0 = 0, nsl = 0, U = 0, C = 1;
    const int G = p.groups;
    if (p.has_mid) {
        const int Z = p.B * p.Hkv;
        U = p.cu_units ? p.cu_units[Z] : Z * p.units_per_z;
        C = p.n_ctas < U ? p.n_ctas : U;
        zb = p.cu_units ? p.cu_units[z] : z * p.units_per_z;
        ze = p.cu_units ? p.cu_units[z + 1] : (z + 1) * p.units_per_z;
        if (ze > zb && C > 0) {
            c0 = cta_of_unit(zb, C, U);
            nsl = (cta_of_unit(ze - 1, C, U) - c0 + 1) * G;
        }
    }
    // Candidate partial j: middle CTA c0 + j / G, consumer group j % G, which
    // stored its partial of this row at the first unit of the row it
    // processed (units ub + g, ub + g + G, ... of the CTA's range), if any.
    auto slot_of = [&](int j) {
        const int c = c0 + j / G, g = j % G;
        const int ub = (int)((int64_t)c * U / C), ue = (int)((int64_t)(c + 1) * U / C);
        const int u0 = zb > ub ? zb : ub;
        const int u = u0 + ((g - (u0 - ub)) % G + G) % G;
        return (u < ze && u < ue) ? u : -1;
    };
    if (tid < (nsl < kFinSlots ? nsl : kFinSlots)) sslot[tid] = slot_of(tid);
    __syncthreads();   // FP statistics complete (FP path), first slots known
    if (p.has_mid && tid < ROWS) { m_row[tid] = fp_ml.x; l_row[tid] = fp_ml.y; }
    __syncthreads();
    for (int j0 = 0; j0 < nsl; j0 += kFinSlots) {
        const int nj = (nsl - j0) < kFinSlots ? (nsl - j0) : kFinSlots;
        if (j0 > 0) {
            __syncthreads();
            if (tid < nj) sslot[tid] = slot_of(j0 + tid);
            __syncthreads();
        }
        // outputs of the first PRE partials are requested together with the
        // statistics: one memory round trip for the usual handful of partials
        float2 pre[PRE][OUTS];
#pragma unroll
        for (int j = 0; j < PRE; ++j)
#pragma unroll
            for (int k = 0; k < OUTS; ++k) {
                const int i = tid + k * kFinThreads;
                pre[j][k] = make_float2(0.f, 0.f);
                const int sl_j = j < nj ? sslot[j] : -1;
                if (sl_j >= 0 && i < rows * D2) {
                    const int r = i / D2, d2 = i % D2;
                    pre[j][k] = *reinterpret_cast<const float2*>(p.ws_o + ((int64_t)sl_j * rows + r) * D + 2 * d2);
                }
            }
        for (int i = tid; i < nj * rows; i += kFinThreads) {
            const int j = i / rows, r = i % rows;
            const int sl_j = sslot[j];
            const float2 ml = sl_j >= 0 ? *reinterpret_cast<const float2*>(p.ws_ml + ((int64_t)sl_j * rows + r) * 2)
                                        : make_float2(-INFINITY, 0.f);
            sw[j * ROWS + r] = ml.x;
            sl[j * ROWS + r] = ml.y;
        }
        __syncthreads();
        if (tid < rows) {
            const int r = tid;
            const float mold = m_row[r];
            float mx = mold;
            for (int j = 0; j < nj; ++j) mx = fmaxf(mx, sw[j * ROWS + r]);
            const float corr = (mold == -INFINITY) ? 0.f : ex2(mold - mx);
            float Ls = l_row[r] * corr;
            for (int j = 0; j < nj; ++j) {
                const float ms = sw[j * ROWS + r];
                const float w = (ms == -INFINITY) ? 0.f : ex2(ms - mx);
                Ls += w * sl[j * ROWS + r];
                sw[j * ROWS + r] = w;
            }
            m_row[r] = mx;
            l_row[r] = Ls;
            c_row[r] = corr;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < OUTS; ++k) {
            const int i = tid + k * kFinThreads;
            if (i >= rows * D2) continue;
            const int r = i / D2, d2 = i % D2;
            const float corr = c_row[r];
            float a0 = acc_m[k][0] * corr, a1 = acc_m[k][1] * corr;
            acc_f[k][0] *= corr;
            acc_f[k][1] *= corr;
#pragma unroll
            for (int j = 0; j < PRE; ++j) {
                if (j >= nj) break;
                const float w = sw[j * ROWS + r];
                a0 = fmaf(w, pre[j][k].x, a0);
                a1 = fmaf(w, pre[j][k].y, a1);
            }
            for (int j = PRE; j < nj; ++j) {
                const float w = sw[j * ROWS + r];
                if (w == 0.f) continue;   // also every missing slot
                const float2 ov = *reinterpret_cast<const float2*>(p.ws_o + ((int64_t)sslot[j] * rows + r) * D + 2 * d2);
                a0 = fmaf(w, ov.x, a0);
                a1 = fmaf(w, ov.y, a1);
            }
            acc_m[k][0] = a0;
            acc_m[k][1] = a1;
        }
    }
    __syncthreads();
    if (tid < rows) f_row[tid] = l_row[tid] > 0.f ? 1.f / l_row[tid] : 0.f;
    if (p.rotation && nsl > 0) {
        // middle part is in the rotated basis: mid @ R (rows via shared memory)
        float* msm = reinterpret_cast<float*>(fsm + L::K_OFF);
#pragma unroll
        for (int k = 0; k < OUTS; ++k) {
            const int i = tid + k * kFinThreads;
            if (i < rows * D2) { msm[2 * i] = acc_m[k][0]; msm[2 * i + 1] = acc_m[k][1]; }
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < OUTS; ++k) {
            const int i = tid + k * kFinThreads;
            if (i >= rows * D2) continue;
            const int r = i / D2, d2 = i % D2;
            float a0 = 0.f, a1 = 0.f;
            for (int e = 0; e < D; ++e) {
                const float mv = msm[r * D + e];
                const float2 rr = *reinterpret_cast<const float2*>(p.rotation + (int64_t)e * D + 2 * d2);
                a0 = fmaf(mv, rr.x, a0);
                a1 = fmaf(mv, rr.y, a1);
            }
            acc_m[k][0] = a0;
            acc_m[k][1] = a1;
        }
    }
    __syncthreads();
    auto* out = reinterpret_cast<T*>(p.out);
#pragma unroll
    for (int k = 0; k < OUTS; ++k) {
        const int i = tid + k * kFinThreads;
        if (i >= rows * D2) continue;
        const int r = i / D2, d2 = i % D2;
        const float inv = f_row[r];
        const int j = r / p.n_q, sq = r % p.n_q;
        T* o = out + (int64_t)b * p.o_sb + (int64_t)(h * p.g + j) * p.o_sh + (int64_t)sq * p.o_ss + 2 * d2;
        o[0] = Elem<DT>::from_f((acc_f[k][0] + acc_m[k][0]) * inv);
        o[1] = Elem<DT>::from_f((acc_f[k][1] + acc_m[k][1]) * inv);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

// Packed code rows (row_bytes = 16..128 per token) are addressed as 128-byte
// rows holding 128/row_bytes tokens each: one stage (kStageTokens tokens) is a
// box of row_bytes 128-byte rows, copied with the 128B swizzle.  Narrower
// boxes (one 64- or 32-byte row per token) made the copy engine issue small
// requests and capped the stream well below HBM bandwidth.
static int make_row_map(CUtensorMap* m, const void* base, int64_t n_rows, int row_bytes) {
    auto enc = encode_fn();
    if (!enc) return FADE_ERR_CUDA;
    if (row_bytes != 16 && row_bytes != 32 && row_bytes != 64 && row_bytes != 128) return FADE_ERR_UNSUPPORTED;
    if ((n_rows * row_bytes) % 128 != 0) return FADE_ERR_ALIGN;
    cuuint64_t dims[2] = {128, (cuuint64_t)(n_rows * row_bytes / 128)};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {128, (cuuint32_t)(kStageTokens * row_bytes / 128)};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box,
                     estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? FADE_OK : FADE_ERR_ALIGN;
}

// V scales: per-token -> 1-D map over rows (box = one stage of rows);
// grouped -> 2-D map [groups][D] (box = the stage's groups).  UINT16 elements:
// the bits are copied, not converted.
static int make_scale_map(CUtensorMap* m, const void* base, int64_t n_rows, bool grouped, int D, int G) {
    auto enc = encode_fn();
    if (!enc) return FADE_ERR_CUDA;
    CUresult r;
    if (!grouped) {
        cuuint64_t dims[1] = {(cuuint64_t)n_rows};
        cuuint64_t strides[1] = {2};
        cuuint32_t box[1] = {(cuuint32_t)kStageTokens};
        cuuint32_t estr[1] = {1};
        r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 1, const_cast<void*>(base), dims, strides + 1, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const int64_t n_groups = (n_rows + G - 1) / G;
        cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)n_groups};
        cuuint64_t strides[1] = {(cuuint64_t)D * 2};
        cuuint32_t box[2] = {(cuuint32_t)D, (cuuint32_t)(kStageTokens / G)};
        cuuint32_t estr[2] = {1, 1};
        r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    return r == CUDA_SUCCESS ? FADE_OK : FADE_ERR_ALIGN;
}

static int sm_count() {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
}

struct MidKernelInfo {
    void* fn;
    int smem;
    int occ;
    int threads;
    int groups;
};

// Function attributes are per device: configure each (kernel, device) once.
constexpr int kMaxDevices = 64;

template <int DT, int D, int KB, int VB, bool VG, int NT, bool QS>
static MidKernelInfo mid_info() {
    static MidKernelInfo info[kMaxDevices] = {};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) dev = 0;
    std::lock_guard<std::mutex> lock(mu);
    MidKernelInfo& i = info[dev];
    if (!i.fn) {
        i.smem = MidLayout<D, KB, VB, VG, NT>::SMEM_BYTES;
        cudaFuncSetAttribute(&middle_kernel<DT, D, KB, VB, VG, NT, QS>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, i.smem);
        int occ = 0;
        i.threads = mid_threads(NT);
        i.groups = mid_groups(NT);
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, &middle_kernel<DT, D, KB, VB, VG, NT, QS>,
                                                      i.threads, i.smem);
        i.occ = occ > 0 ? occ : 1;
        i.fn = reinterpret_cast<void*>(&middle_kernel<DT, D, KB, VB, VG, NT, QS>);
    }
    return i;
}

template <int DT, int D, int NT>
static MidKernelInfo select_mid(int kb, int vb, bool vg, bool rot) {
    if (!rot && kb == 4 && vb == 4 && !vg) return mid_info<DT, D, 4, 4, false, NT, false>();
    if (!rot && kb == 4 && vb == 2 && vg) return mid_info<DT, D, 4, 2, true, NT, false>();
    if (rot && kb == 4 && vb == 4 && !vg) return mid_info<DT, D, 4, 4, false, NT, true>();
    if (rot && kb == 2 && vb == 2 && !vg) return mid_info<DT, D, 2, 2, false, NT, true>();
    return MidKernelInfo{nullptr, 0, 0, 0, 0};
}

template <int DT, int NT>
static MidKernelInfo mid_tc_info() {
    static MidKernelInfo info[kMaxDevices] = {};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) dev = 0;
    std::lock_guard<std::mutex> lock(mu);
    MidKernelInfo& i = info[dev];
    if (!i.fn) {
        i.smem = TcLayout::SMEM_BYTES;
        cudaFuncSetAttribute(&middle_tc_kernel<DT, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, i.smem);
        int occ = 0;
        i.threads = kTcThreads;
        i.groups = 1;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, &middle_tc_kernel<DT, NT>, i.threads, i.smem);
        i.occ = occ > 0 ? occ : 1;
        i.fn = reinterpret_cast<void*>(&middle_tc_kernel<DT, NT>);
    }
    return i;
}

// Middle-kernel family for INT4 K and V at D = 128: 0 = mma.sync (default,
// the faster one on B200), 1 = tcgen05 (fade_set_middle_kernel).  Read when a
// call builds its plan; process-wide.
static std::atomic<int> g_middle_kernel{0};

template <int DT>
static MidKernelInfo select_mid_d(int D, int NT, int kb, int vb, bool vg, bool rot) {
    if (g_middle_kernel.load(std::memory_order_relaxed) == 1 && D == 128 && !rot && kb == 4 && vb == 4 && !vg)
        return NT == 1 ? mid_tc_info<DT, 1>() : mid_tc_info<DT, 2>();
    if (D == 128) return NT == 1 ? select_mid<DT, 128, 1>(kb, vb, vg, rot) : select_mid<DT, 128, 2>(kb, vb, vg, rot);
    if (D == 64) return NT == 1 ? select_mid<DT, 64, 1>(kb, vb, vg, rot) : select_mid<DT, 64, 2>(kb, vb, vg, rot);
    return MidKernelInfo{nullptr, 0, 0, 0, 0};
}

struct FinKernelInfo {
    void* fn;
    int smem;
};

template <int DT, int D, int NT>
static FinKernelInfo fin_info() {
    static FinKernelInfo info[kMaxDevices] = {};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= kMaxDevices) dev = 0;
    std::lock_guard<std::mutex> lock(mu);
    FinKernelInfo& i = info[dev];
    if (!i.fn) {
        i.smem = FinLayout<D, NT>::BYTES;
        cudaFuncSetAttribute(&finish_kernel<DT, D, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, i.smem);
        i.fn = reinterpret_cast<void*>(&finish_kernel<DT, D, NT>);
    }
    return i;
}

template <int DT>
static FinKernelInfo select_fin(int D, int NT) {
    if (D == 128) return NT == 1 ? fin_info<DT, 128, 1>() : fin_info<DT, 128, 2>();
    if (D == 64) return NT == 1 ? fin_info<DT, 64, 1>() : fin_info<DT, 64, 2>();
    return FinKernelInfo{nullptr, 0};
}

struct Plan {
    int rows, NT, g;
    int mid_idx;         // index of the quantised segment or -1
    int kb, vb;
    bool vg;
    int units_per_z;     // uniform
    int64_t max_units;   // sizing bound
    int n_ctas;
    int n_fp;
    size_t off_err, off_qrot, off_age, off_fpml, off_fpo, off_ml, off_o, total;
    MidKernelInfo mk;
};

static int make_plan(const fade_decode_desc* d, Plan* pl) {
    if (!d) return FADE_ERR_INVALID_ARG;
    if (d->dtype != FADE_F16 && d->dtype != FADE_BF16) return FADE_ERR_UNSUPPORTED;
    if (d->B < 0 || d->Hq <= 0 || d->Hkv <= 0 || d->D <= 0 || d->n_q <= 0) return FADE_ERR_INVALID_ARG;
    if (d->Hq % d->Hkv != 0) return FADE_ERR_INVALID_ARG;
    if (d->D != 64 && d->D != 128) return FADE_ERR_UNSUPPORTED;
    if (d->n_segments < 0 || d->n_segments > FADE_MAX_SEGMENTS) return FADE_ERR_INVALID_ARG;
    pl->g = d->Hq / d->Hkv;
    pl->rows = pl->g * d->n_q;
    if (pl->rows > 16) return FADE_ERR_UNSUPPORTED;
    pl->NT = pl->rows > 8 ? 2 : 1;
    pl->mid_idx = -1;
    pl->n_fp = 0;
    for (int i = 0; i < d->n_segments; ++i) {
        const fade_kv_segment& s = d->seg[i];
        if (s.kind == FADE_SEG_FP) {
            if (!s.k || !s.v) return FADE_ERR_INVALID_ARG;
            ++pl->n_fp;
            continue;
        }
        if (pl->mid_idx >= 0) return FADE_ERR_UNSUPPORTED;  // one quantised tier per call
        pl->mid_idx = i;
        if (s.kind == FADE_SEG_INT4) { pl->kb = 4; pl->vb = 4; pl->vg = false; }
        else if (s.kind == FADE_SEG_INT4K_INT2V) {
            pl->kb = 4; pl->vb = 2; pl->vg = true;
            if (s.group < 16 || s.group > kStageTokens || kStageTokens % s.group != 0) return FADE_ERR_UNSUPPORTED;
        } else if (s.kind == FADE_SEG_ROT) {
            if (s.bits != 2 && s.bits != 4) return FADE_ERR_UNSUPPORTED;
            pl->kb = s.bits; pl->vb = s.bits; pl->vg = false;
            if (!d->rotation) return FADE_ERR_INVALID_ARG;
            if (!aligned16(d->rotation)) return FADE_ERR_ALIGN;   // R is staged with 16-byte loads
        } else return FADE_ERR_INVALID_ARG;
        if (!s.k || !s.v || !s.k_scale || !s.v_scale) return FADE_ERR_INVALID_ARG;
        if (!aligned16(s.k) || !aligned16(s.v)) return FADE_ERR_ALIGN;
        if (s.lens && s.max_len <= 0 && !d->cu_units) return FADE_ERR_INVALID_ARG;
        if (s.page_table && (s.pages_per_row <= 0 || s.n_rows <= 0)) return FADE_ERR_INVALID_ARG;
    }
    const int Z = d->B * d->Hkv;
    pl->units_per_z = 0;
    pl->max_units = 0;
    pl->n_ctas = 0;
    if (pl->mid_idx >= 0 && Z > 0) {
        const fade_kv_segment& s = d->seg[pl->mid_idx];
        const int64_t ml = s.lens ? s.max_len : s.len;
        const int64_t upz = (ml + kStageTokens - 1) / kStageTokens;
        pl->units_per_z = (int)upz;
        pl->max_units = upz * Z;
        int dt = d->dtype;
        const bool rot = s.kind == FADE_SEG_ROT;
        pl->mk = dt == FADE_F16 ? select_mid_d<FADE_F16>(d->D, pl->NT, pl->kb, pl->vb, pl->vg, rot)
                                : select_mid_d<FADE_BF16>(d->D, pl->NT, pl->kb, pl->vb, pl->vg, rot);
        if (!pl->mk.fn) return FADE_ERR_UNSUPPORTED;
        int C = d->n_ctas > 0 ? d->n_ctas : sm_count() * pl->mk.occ;
        if (!d->cu_units && pl->max_units < C) C = (int)pl->max_units;
        if (C < 1) C = 1;
        pl->n_ctas = C;
    }
    const bool rot = pl->mid_idx >= 0 && d->seg[pl->mid_idx].kind == FADE_SEG_ROT;
    size_t off = 0;
    pl->off_err = off; off += 256;
    pl->off_qrot = off;
    if (rot) off += ((size_t)d->B * d->Hq * d->n_q * d->D * 4 + 255) / 256 * 256;
    pl->off_age = off; off += ((size_t)Z * 4 + 255) / 256 * 256;
    pl->off_fpml = off; off += ((size_t)Z * pl->rows * 2 * 4 + 255) / 256 * 256;
    pl->off_fpo = off; off += ((size_t)Z * pl->rows * d->D * 4 + 255) / 256 * 256;
    pl->off_ml = off; off += ((size_t)pl->max_units * pl->rows * 2 * 4 + 255) / 256 * 256;
    pl->off_o = off; off += (size_t)pl->max_units * pl->rows * d->D * 4;
    pl->total = off;
    return FADE_OK;
}

// The query rotation stages R (up to 64 KB) in shared memory: opt in once per
// device and kernel instantiation.
static cudaError_t rotate_queries_smem_attr(const void* fn, int which) {
    static bool done[kMaxDevices][4] = {};
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) dev = 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev][which]) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (128 * 128 + 128 * kRotQS) * 4);
        if (e != cudaSuccess) return e;
        done[dev][which] = true;
    }
    return cudaSuccess;
}

static cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace fade

using namespace fade;

extern "C" size_t fade_decode_attn_workspace_size(const fade_decode_desc* d) {
    Plan pl;
    if (make_plan(d, &pl) != FADE_OK) return 0;
    return pl.total;
}

static int decode_attn_impl(const fade_decode_desc* d, const fade_age_out_desc* a, void* workspace,
                            size_t ws_bytes, void* stream) {
    Plan pl;
    int st = make_plan(d, &pl);
    if (st != FADE_OK) return st;
    if (a) {
        if (a->ring_seg < 0 || a->ring_seg >= d->n_segments || a->mid_seg < 0 || a->mid_seg >= d->n_segments)
            return FADE_ERR_INVALID_ARG;
        const fade_kv_segment& rg = d->seg[a->ring_seg];
        const fade_kv_segment& md = d->seg[a->mid_seg];
        if (rg.kind != FADE_SEG_FP || md.kind != FADE_SEG_INT4) return FADE_ERR_UNSUPPORTED;
        if (d->n_q != 1 || !a->k_new || !a->v_new || !md.lens || md.max_len <= 0) return FADE_ERR_INVALID_ARG;
        if (rg.lens || rg.len != a->ring_cap || a->ring_cap <= 0) return FADE_ERR_INVALID_ARG;
        if (md.page_table) return FADE_ERR_UNSUPPORTED;   // the age-out writes dense rows
    }
    if (d->B == 0) return FADE_OK;
    if (!d->q || !d->out) return FADE_ERR_INVALID_ARG;
    if (!workspace || ws_bytes < pl.total) return FADE_ERR_WORKSPACE;
    cudaStream_t s = as_stream(stream);
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    const int Z = d->B * d->Hkv;
    const bool has_mid = pl.mid_idx >= 0 && pl.max_units > 0;
    const bool rot = has_mid && d->seg[pl.mid_idx].kind == FADE_SEG_ROT;
    float* qrot = reinterpret_cast<float*>(ws + pl.off_qrot);
    const float qk_scale = d->sm_scale * kLog2e;

    if (rot) {
        const bool f16 = d->dtype == FADE_F16, d64 = d->D == 64;
        void* fn = f16 ? (d64 ? (void*)&rotate_queries_kernel<FADE_F16, 64> : (void*)&rotate_queries_kernel<FADE_F16, 128>)
                       : (d64 ? (void*)&rotate_queries_kernel<FADE_BF16, 64> : (void*)&rotate_queries_kernel<FADE_BF16, 128>);
        const void* qp = d->q;
        int Hq = d->Hq, nq = d->n_q, D = d->D;
        int64_t a = d->q_sb, b2 = d->q_sh, c2 = d->q_ss;
        const float* R = d->rotation;
        int n_rows = d->B * d->Hq * d->n_q;
        void* args[] = {(void*)&qp, &Hq, &nq, &a, &b2, &c2, (void*)&R, (void*)&qrot, &n_rows};
        const size_t rsmem = (size_t)(D * D + D * kRotQS) * 4;
        FADE_CUDA_TRY(rotate_queries_smem_attr(fn, (f16 ? 0 : 2) + (d64 ? 0 : 1)));
        FADE_CUDA_TRY(launch_pdl(fn, dim3((unsigned)((n_rows + kRotRows - 1) / kRotRows)), dim3((unsigned)(2 * D)),
                                 rsmem, s, args));
    }
    if (has_mid) {
        const fade_kv_segment& sg = d->seg[pl.mid_idx];
        CUtensorMap tk, tv;
        const int rbk = d->D * pl.kb / 8, rbv = d->D * pl.vb / 8;
        // Rows the maps may address: reads past this extent are zero-filled by
        // the TMA unit (and masked), never fetched from beyond the allocation.
        const int64_t maxlen = sg.lens ? sg.max_len : sg.len;
        int64_t n_rows = sg.n_rows;
        if (n_rows <= 0) {
            if (sg.row_base || sg.page_table) return FADE_ERR_INVALID_ARG;
            n_rows = (int64_t)(d->B - 1) * sg.row_sb + (int64_t)(d->Hkv - 1) * sg.row_sh + maxlen;
        }
        if (n_rows <= 0) n_rows = 1;
        if (n_rows >= ((int64_t)1 << 31)) return FADE_ERR_UNSUPPORTED;
        // every (b, h) segment must start on a 128-byte row of both code arrays
        {
            const int tpr = 128 / (rbk < rbv ? rbk : rbv);
            if (sg.row_sb % tpr || sg.row_sh % tpr) return FADE_ERR_ALIGN;
        }
        if ((st = make_row_map(&tk, sg.k, n_rows, rbk)) != FADE_OK) return st;
        if ((st = make_row_map(&tv, sg.v, n_rows, rbv)) != FADE_OK) return st;
        // V scales by TMA when every stage's first row lands on a 16-byte
        // boundary of the scale array; otherwise the producer warp loads them.
        CUtensorMap ts;
        memset(&ts, 0, sizeof(ts));
        int scale_tma = aligned16(sg.v_scale) && !sg.row_base;
        if (scale_tma && !pl.vg) scale_tma = (sg.row_sb % 8 == 0) && (sg.row_sh % 8 == 0);
        if (scale_tma && pl.vg) scale_tma = (d->D * 2) % 16 == 0;
        if (scale_tma && make_scale_map(&ts, sg.v_scale, n_rows, pl.vg, d->D, pl.vg ? sg.group : 1) != FADE_OK)
            scale_tma = 0;
        MidParams mp = {};
        mp.dtype = d->dtype;
        mp.B = d->B; mp.Hq = d->Hq; mp.Hkv = d->Hkv; mp.D = d->D; mp.n_q = d->n_q;
        mp.g = pl.g; mp.rows = pl.rows;
        mp.qk_scale = qk_scale;
        if (rot) {
            mp.q = qrot; mp.q_is_f32 = 1;
            mp.q_ss = d->D; mp.q_sh = (int64_t)d->n_q * d->D; mp.q_sb = (int64_t)d->Hq * d->n_q * d->D;
        } else {
            mp.q = d->q; mp.q_is_f32 = 0;
            mp.q_sb = d->q_sb; mp.q_sh = d->q_sh; mp.q_ss = d->q_ss;
        }
        mp.k_scale = sg.k_scale; mp.ks_sb = sg.ks_sb; mp.ks_sh = sg.ks_sh;
        mp.v_scale = sg.v_scale;
        mp.group = pl.vg ? sg.group : 0;
        mp.row_sb = sg.row_sb; mp.row_sh = sg.row_sh; mp.row_base = sg.row_base;
        mp.lens = sg.lens; mp.len = sg.len;
        mp.cu_units = d->cu_units;
        mp.page_table = sg.page_table;
        mp.pages_per_row = sg.pages_per_row;
        mp.units_per_z = pl.units_per_z;
        mp.n_ctas = pl.n_ctas;
        mp.ws_ml = reinterpret_cast<float*>(ws + pl.off_ml);
        mp.ws_o = reinterpret_cast<float*>(ws + pl.off_o);
        mp.ws_err = reinterpret_cast<int*>(ws + pl.off_err);
        mp.scale_tma = scale_tma;
        mp.early = (a && a->prefetch_tiers) ? 1 : 0;
        // FP tiers for the FP warp
        mp.n_fp = 0;
        for (int i = 0; i < d->n_segments; ++i) {
            const fade_kv_segment& f = d->seg[i];
            if (f.kind != FADE_SEG_FP) continue;
            FpSeg& o = mp.fp[mp.n_fp++];
            o.k = f.k; o.v = f.v; o.row_sb = f.row_sb; o.row_sh = f.row_sh;
            o.row_base = f.row_base; o.lens = f.lens; o.len = f.len;
            // fragments are read with 16-byte (K) and 8-byte (V) loads
            if (!aligned16(f.k) || !aligned16(f.v)) return FADE_ERR_ALIGN;
        }
        mp.qo = d->q; mp.qo_sb = d->q_sb; mp.qo_sh = d->q_sh; mp.qo_ss = d->q_ss;
        mp.ws_fpml = reinterpret_cast<float*>(ws + pl.off_fpml);
        mp.ws_fpo = reinterpret_cast<float*>(ws + pl.off_fpo);
        mp.ws_age = reinterpret_cast<int*>(ws + pl.off_age);
        if (a) {
            mp.age = 1;
            mp.ring_fp = 0;
            for (int i = 0; i < a->ring_seg; ++i) mp.ring_fp += d->seg[i].kind == FADE_SEG_FP ? 1 : 0;
            mp.ring_cap = a->ring_cap;
            mp.ring_origin = a->ring_origin;
            mp.k_new = a->k_new; mp.v_new = a->v_new; mp.new_sb = a->new_sb; mp.new_sh = a->new_sh;
            // the FP warp stages the new token with 16-byte copies
            if (!aligned16(a->k_new) || !aligned16(a->v_new) || (a->new_sb * 2) % 16 || (a->new_sh * 2) % 16)
                return FADE_ERR_ALIGN;
            mp.mid_cap = sg.max_len;
            mp.mid_len = sg.lens;
            mp.age_k = reinterpret_cast<uint8_t*>(const_cast<void*>(sg.k));
            mp.age_v = reinterpret_cast<uint8_t*>(const_cast<void*>(sg.v));
        }
        mp.q_vec = aligned16(sg.k_scale) && sg.ks_sb % 8 == 0 && sg.ks_sh % 8 == 0 &&
                   (rot || (aligned16(d->q) && d->q_sb % 8 == 0 && d->q_sh % 8 == 0 && d->q_ss % 8 == 0));
        void* args[] = {(void*)&tk, (void*)&tv, (void*)&ts, (void*)&mp};
        FADE_CUDA_TRY(launch_pdl(pl.mk.fn, dim3((unsigned)pl.n_ctas), dim3((unsigned)pl.mk.threads),
                                 (size_t)pl.mk.smem, s, args));
    }
    // Finisher: FP tiers + merge of the middle partials -> out.  Always
    // launched (it also writes rows whose middle is empty).
    FinParams fp = {};
    fp.B = d->B; fp.Hq = d->Hq; fp.Hkv = d->Hkv; fp.D = d->D; fp.n_q = d->n_q;
    fp.g = pl.g; fp.rows = pl.rows; fp.qk_scale = qk_scale;
    fp.q = d->q; fp.q_sb = d->q_sb; fp.q_sh = d->q_sh; fp.q_ss = d->q_ss;
    fp.out = d->out; fp.o_sb = d->o_sb; fp.o_sh = d->o_sh; fp.o_ss = d->o_ss;
    fp.vec = 1;
    for (int i = 0; i < d->n_segments; ++i) {
        const fade_kv_segment& sg = d->seg[i];
        if (sg.kind != FADE_SEG_FP) continue;
        FpSeg& f = fp.fp[fp.n_fp++];
        f.k = sg.k; f.v = sg.v; f.row_sb = sg.row_sb; f.row_sh = sg.row_sh;
        f.row_base = sg.row_base; f.lens = sg.lens; f.len = sg.len;
        if (!aligned16(sg.k) || !aligned16(sg.v)) fp.vec = 0;
    }
    if ((d->D * 2) % 16 != 0) fp.vec = 0;
    fp.has_mid = has_mid ? 1 : 0;
    fp.cu_units = d->cu_units;
    fp.units_per_z = pl.units_per_z;
    fp.n_ctas = pl.n_ctas;
    fp.groups = has_mid ? pl.mk.groups : 1;
    fp.ws_ml = reinterpret_cast<const float*>(ws + pl.off_ml);
    fp.ws_o = reinterpret_cast<const float*>(ws + pl.off_o);
    fp.rotation = rot ? d->rotation : nullptr;
    fp.ws_fpml = reinterpret_cast<const float*>(ws + pl.off_fpml);
    fp.ws_fpo = reinterpret_cast<const float*>(ws + pl.off_fpo);
    fp.ws_age = reinterpret_cast<const int*>(ws + pl.off_age);
    if (a) {
        fp.age = 1;
        fp.mid_len = const_cast<int32_t*>(d->seg[a->mid_seg].lens);
    }
    const FinKernelInfo fk = d->dtype == FADE_F16 ? select_fin<FADE_F16>(d->D, pl.NT)
                                                  : select_fin<FADE_BF16>(d->D, pl.NT);
    if (!fk.fn) return FADE_ERR_UNSUPPORTED;
    void* fargs[] = {(void*)&fp};
    FADE_CUDA_TRY(launch_pdl(fk.fn, dim3((unsigned)Z), dim3(kFinThreads), (size_t)fk.smem, s, fargs));
    return FADE_OK;
}

extern "C" int fade_decode_attn(const fade_decode_desc* d, void* workspace, size_t ws_bytes,
                                void* stream) {
    return decode_attn_impl(d, nullptr, workspace, ws_bytes, stream);
}

extern "C" int fade_decode_attn_age_out(const fade_decode_desc* d, const fade_age_out_desc* a,
                                        void* workspace, size_t ws_bytes, void* stream) {
    if (!a) return FADE_ERR_INVALID_ARG;
    return decode_attn_impl(d, a, workspace, ws_bytes, stream);
}

extern "C" int fade_workspace_check(void* workspace, size_t ws_bytes, void* stream) {
    if (!workspace || ws_bytes < 256) return FADE_ERR_WORKSPACE;
    int h = 0;
    cudaStream_t s = as_stream(stream);
    FADE_CUDA_TRY(cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, s));
    FADE_CUDA_TRY(cudaStreamSynchronize(s));
    if (h != 0) {
        FADE_CUDA_TRY(cudaMemsetAsync(workspace, 0, 256, s));
        FADE_CUDA_TRY(cudaStreamSynchronize(s));
        return FADE_ERR_TIMEOUT;
    }
    return FADE_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of fade_decode_attn.
//
// Some callers cannot allocate device memory at the point where they run
// attention: code inside an allocator-free serving runtime that was handed a
// fixed memory pool, plugin hosts whose policy forbids cudaMalloc after
// start-up, or callers that cannot hold a workspace object across calls.
// This entry point takes its scratch space from a fixed array compiled into
// the library instead of a caller-supplied workspace.
// ---------------------------------------------------------------------------
namespace fade {
// Every GPU that loads the library reserves this array until the process exits.
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
// Device address of the array per device.  In host code the symbol itself is
// only a host-side stand-in, so the address is looked up once per device.
static void* g_noalloc_ptr[kMaxDevices] = {};
static std::mutex g_noalloc_mu;

static int noalloc_scratch(void** out) {
    int dev = 0;
    FADE_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return FADE_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        FADE_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return FADE_OK;
}
}  // namespace fade

extern "C" size_t fade_decode_attn_noalloc_max_bytes(void) { return fade::kNoAllocScratchBytes; }

extern "C" int fade_decode_attn_noalloc(const fade_decode_desc* d, void* stream) {
    const size_t need = fade_decode_attn_workspace_size(d);
    if (need == 0) {
        Plan pl;
        const int st = make_plan(d, &pl);
        return st != FADE_OK ? st : FADE_ERR_INVALID_ARG;
    }
    if (need > fade::kNoAllocScratchBytes) return FADE_ERR_WORKSPACE;
    void* ws = nullptr;
    int st = fade::noalloc_scratch(&ws);
    if (st != FADE_OK) return st;
    // The array keeps the previous call's bytes.  Every partial, statistic
    // and age-out length the kernels read is written earlier in the same
    // call; the only word that must start at zero is the error word, which
    // is zero when the library loads and is cleared again by
    // fade_decode_attn_noalloc_check after it reports a timeout (so a timeout
    // stays visible until the caller asks for it, as with a workspace).
    return fade_decode_attn(d, ws, fade::kNoAllocScratchBytes, stream);
}

extern "C" int fade_set_middle_kernel(int kind) {
    if (kind != 0 && kind != 1) return FADE_ERR_INVALID_ARG;
    fade::g_middle_kernel.store(kind, std::memory_order_relaxed);
    return FADE_OK;
}

extern "C" int fade_get_middle_kernel(void) { return fade::g_middle_kernel.load(std::memory_order_relaxed); }

extern "C" int fade_decode_attn_noalloc_check(void* stream) {
    void* ws = nullptr;
    const int st = fade::noalloc_scratch(&ws);
    if (st != FADE_OK) return st;
    return fade_workspace_check(ws, fade::kNoAllocScratchBytes, stream);
}
