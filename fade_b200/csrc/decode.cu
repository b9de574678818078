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
//   k0  rotate_queries   (only with a rotated tier): q_rot = q @ R^T, fp32.
//   kf  fp_tier_kernel   one CTA per (b, kv-head): attention over the FP
//                        sink/recent tiers -> an un-normalised partial (or the
//                        final output when there is no quantised middle).
//   k1  middle_kernel    persistent stream-K over the quantised middle; every
//                        CTA writes one partial per (b, kv-head) it touched and
//                        counts its arrival; the CTA that completes a row merges
//                        the FP partial with all middle partials and writes `out`.
//
// k1 data path per CTA (5 warps):
//   warp 4 (producer): 2-D TMA (cp.async.bulk.tensor, no multicast) of 128
//     token rows of packed K and V codes into a 4-stage ring, swizzled so the
//     ldmatrix reads below are bank-conflict free; it also stages the V scales
//     (normalised per 32-token slice) with plain loads.  mbarrier full/empty.
//   warps 0-3 (consumers): each owns 32 tokens of a stage.
//     S^T[16 tok x 8 rows] = K_codes[16 x D] . (q*k_scale/qn)^T   (mma.sync
//       m16n8k16 f16 -> f32; the GQA query rows of one kv head are the N dim)
//     codes are turned into exact fp16 integers in registers with the
//     magic-exponent trick (LUT-free int4 -> fp16 conversion, as used in
//     FasterTransformer's mixed-precision GEMMs): (x & mask) ^ (0x6400|sign)
//     makes 1024 + u (or 1024 + 16u), one HADD2 removes the bias.
//     online softmax in log2 space; P (fp16, V scale folded in) is transposed
//     with movmatrix and O^T[D x 8] += V_codes^T . P^T (mma.sync again).
//   The channel order inside a thread is permuted to match the packed layout;
//   q fragments are built with the same permutation, so nothing is shuffled.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace fade {

// Ablation switch for profiling builds only (default 0 = full kernel):
// 1 = consumers only cycle the pipeline, 2 = QK^T only, 3 = no scale multiply,
// 4 = as 1 without the L2 cache hint, 5 = as 1 without the scale copy,
// 6 = as 1 without per-row setup / flush / merge.
#ifndef FADE_ABLATE
#define FADE_ABLATE 0
#endif
// Timeline tracing for profiling builds only (FADE_TRACE defined): per CTA
// event timestamps into a device array read back by fade_trace_read().
#ifdef FADE_TRACE
constexpr int kTraceEv = 96;
__device__ unsigned long long g_trace[1024 * kTraceEv];
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
#define FADE_TR(slot) do { if (threadIdx.x == 0 && blockIdx.x < 1024 && (slot) < kTraceEv) g_trace[blockIdx.x * kTraceEv + (slot)] = gtimer(); } while (0)
#define FADE_TRP(slot) do { if (threadIdx.x == kConsumerWarps * 32 && blockIdx.x < 1024 && (slot) < kTraceEv) g_trace[blockIdx.x * kTraceEv + (slot)] = gtimer(); } while (0)
#else
#define FADE_TR(slot) do {} while (0)
#define FADE_TRP(slot) do {} while (0)
#endif
constexpr int kConsumerWarps = 4;
constexpr int kMidThreads = (kConsumerWarps + 1) * 32;
constexpr int kStageTokens = 128;  // 32 tokens per consumer warp
constexpr int kStages = 4;
constexpr int kFpThreads = 256;
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint32_t kWaitLimit = 1u << 22;  // bounded mbarrier polling

// ---------------------------------------------------------------------------
// PTX wrappers (mbarrier, TMA, ldmatrix, movmatrix, mma)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
        : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
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
    if (*abort_flag) return false;
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 1023u) == 1023u && *abort_flag) return false;
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
        if (FADE_ABLATE == 3) return a ^ (b & 1u);
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
        if (FADE_ABLATE == 3) return a ^ (b & 1u);
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
template <int DT> struct Conv {
    // INT4: bytes b0..b3 of x hold elements (2j: high nibble, 2j+1: low).
    // h[0]=(e1,e5) h[1]=(e0,e4) h[2]=(e3,e7) h[3]=(e2,e6)
    __device__ __forceinline__ static void int4(uint32_t x, uint32_t (&h)[4]) {
        h[0] = Pk<DT>::sub(lop3_and_xor(x, 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
        h[1] = Pk<DT>::sub(lop3_and_xor(x >> 4, 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
        h[2] = Pk<DT>::sub(lop3_and_xor(x >> 8, 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
        h[3] = Pk<DT>::sub(lop3_and_xor(x >> 12, 0x000F000Fu, Pk<DT>::K4), Pk<DT>::B4);
    }
    // 2-bit: field f of a byte sits at bit 6-2f.  h[0..3] = fields 3,2,1,0 of
    // bytes (0,2); h[4..7] = fields 3,2,1,0 of bytes (1,3).
    __device__ __forceinline__ static void int2(uint32_t x, uint32_t (&h)[8]) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            h[i] = Pk<DT>::sub(lop3_and_xor(x >> (2 * i), 0x00030003u, Pk<DT>::K2), Pk<DT>::B2);
    }
};

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
    int units_per_z;                // uniform case
    int n_ctas;
    float* ws_ml;                   // [U][rows][2]
    float* ws_o;                    // [U][rows][D]
    int* ws_err;
    int* counters;                  // [Z] arrivals per row (zeroed by fp_tier_kernel)
    int scale_tma;                  // V scales arrive by TMA (row starts 8-aligned)
    int q_vec;                      // q / k_scale rows allow 16-byte loads
    const float* fp_ml;             // FP-tier partial [Z][rows][2] or null
    const float* fp_o;              // [Z][rows][D]
    void* out;                      // [B,Hq,n_q,D] model dtype
    int64_t o_sb, o_sh, o_ss;
    const float* rotation;          // rotated middle: out = fp + mid @ R
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
    static constexpr int SC_BASE = kStages * STAGE_BYTES;
    static constexpr int RING_BYTES = SC_BASE + kStages * SC_BYTES;
    static constexpr int OBUF_BYTES = (NT * 8 * D * 4 > 4096) ? NT * 8 * D * 4 : 4096;  // >= merge scratch
    static constexpr int ML_BYTES = kConsumerWarps * 16 * 2 * 4;
    static constexpr int BAR_OFF = RING_BYTES + OBUF_BYTES + ML_BYTES;
    static constexpr int FLAG_OFF = BAR_OFF + 2 * kStages * 8;
    static constexpr int SMEM_BYTES = FLAG_OFF + 16 + 1024;  // +1024 for alignment
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
// k1: middle tier, persistent stream-K
// QSPLIT: the query is fp32 (rotated tiers) and is fed to the MMA as a
// hi + lo pair of model-dtype values (two MMAs per k-step).
// ---------------------------------------------------------------------------
template <int DT, int D, int KB, int VB, bool VGROUP, int NT, bool QSPLIT>
__global__ void __launch_bounds__(kMidThreads, (NT == 1 ? 3 : 1))
middle_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
              const __grid_constant__ CUtensorMap tmap_s, MidParams p) {
    using L = MidLayout<D, KB, VB, VGROUP, NT>;
    using KMap = ChanMap<KB>;
    using VMap = ChanMap<VB>;
    using P = Pk<DT>;
    constexpr int KSTEPS = D / 16;   // k-steps of the QK product
    constexpr int MT = D / 16;       // m-tiles of the PV product (rows = channels)
    constexpr int NQ = QSPLIT ? 2 : 1;

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* obuf = reinterpret_cast<float*>(smem + L::RING_BYTES);
    float* mlbuf = reinterpret_cast<float*>(smem + L::RING_BYTES + L::OBUF_BYTES);
    const uint32_t bar_base = smem_u32(smem + L::BAR_OFF);
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (kStages + s); };

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int Z = p.B * p.Hkv;
    const int U = total_units(p, Z);
    // Never more CTAs than units, so every working CTA owns at least one unit
    // (the merge counts arrivals per row by CTA range).
    const int C = p.n_ctas < U ? p.n_ctas : U;
    const int c = blockIdx.x;
    if (c >= C) return;
    const int ub = (int)((int64_t)c * U / C), ue = (int)((int64_t)(c + 1) * U / C);

    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::FLAG_OFF);
    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full_bar(s), 32);
            mbar_init(empty_bar(s), kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    FADE_TR(0);
    // Inputs may be produced by the previous kernel in the stream (age-out,
    // query rotation): wait for it before touching global memory, then let the
    // next kernel in the stream start its prologue.
    griddep_wait();
    griddep_launch_dependents();
    FADE_TR(1);
    if (ub >= ue) return;

    if (warp == kConsumerWarps) {
        // ------------------------------ producer ------------------------------
        const uint64_t policy = evict_first_policy();
        if (lane == 0) {
            prefetch_tmap(&tmap_k);
            prefetch_tmap(&tmap_v);
            if (p.scale_tma) prefetch_tmap(&tmap_s);
        }
        int z = z_of_unit(p, Z, ub);
        int zb = units_begin(p, z), ze = units_begin(p, z + 1);
        for (int u = ub, i = 0; u < ue; ++u, ++i) {
            while (u >= ze) { ++z; zb = ze; ze = units_begin(p, z + 1); }
            const int s = i % kStages;
            const uint32_t ph = (uint32_t)(i / kStages) & 1u;
            if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.ws_err)) continue;
            const int64_t tok0 = (int64_t)(u - zb) * kStageTokens;
            const int64_t row0 = seg_row0(p, z) + tok0;
            const int64_t len = seg_len(p, z / p.Hkv);
            uint8_t* st = smem + s * L::STAGE_BYTES;
            // Units past this row's length (uniform grid over a capacity bound)
            // carry no tokens: complete the stage without a copy.
            uint8_t* scs = smem + L::SC_BASE + s * L::SC_BYTES;
            FADE_TRP(40 + i);
            if (lane == 0 && tok0 < len) {
                const uint32_t sc_bytes = (p.scale_tma && FADE_ABLATE != 5) ? (uint32_t)L::sc_box_bytes(p.group) : 0u;
                mbar_expect_tx(full_bar(s), (uint32_t)(L::K_BYTES + L::V_BYTES) + sc_bytes);
                // maps address 128-byte rows: token row0 starts at row0*RB/128
#if FADE_ABLATE == 4
                asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                             ::"r"(smem_u32(st + L::K_OFF)), "l"(reinterpret_cast<uint64_t>(&tmap_k)), "r"(0),
                             "r"((int)(row0 * L::RBK / 128)), "r"(full_bar(s)) : "memory");
                asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                             ::"r"(smem_u32(st + L::V_OFF)), "l"(reinterpret_cast<uint64_t>(&tmap_v)), "r"(0),
                             "r"((int)(row0 * L::RBV / 128)), "r"(full_bar(s)) : "memory");
#else
                tma_load_2d(smem_u32(st + L::K_OFF), &tmap_k, 0, (int)(row0 * L::RBK / 128), full_bar(s), policy);
                tma_load_2d(smem_u32(st + L::V_OFF), &tmap_v, 0, (int)(row0 * L::RBV / 128), full_bar(s), policy);
#endif
                if (p.scale_tma && FADE_ABLATE != 5) {
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
        // Drain: wait until the consumers released every stage still in flight,
        // so no TMA write targets this CTA's shared memory after it exits.
        const int n = ue - ub;
        for (int i = (n > kStages ? n : kStages); i < n + kStages; ++i) {
            const int s = i % kStages;
            const uint32_t ph = (uint32_t)(i / kStages) & 1u;
            mbar_wait(empty_bar(s), ph ^ 1u, abort_flag, p.ws_err);
        }
        return;
    }

    // ------------------------------ consumers ------------------------------
    const int gid = lane >> 2, t = lane & 3;
    const int ctid = threadIdx.x;  // 0..127
    uint32_t qf[NQ][NT][KSTEPS][2];  // B fragments (exact model-dtype query)
    uint32_t ksc[KSTEPS][2];         // K scale pairs matching the A pairs
    float m_run[NT][2], l_run[NT][2];
    float o[NT][MT][4];
    int cur_z = -1;
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
#pragma unroll
            for (int cb = 0; cb < KSTEPS * 16 / CHW; ++cb) {
                if constexpr (QSPLIT) {
                    float e[CH];
                    const float* ptr = reinterpret_cast<const float*>(p.q) + qoff + cb * CHW + CH * t;
#pragma unroll
                    for (int c4 = 0; c4 < CH / 4; ++c4) {
                        const float4 v4 = rv ? __ldg(reinterpret_cast<const float4*>(ptr) + c4)
                                             : make_float4(0.f, 0.f, 0.f, 0.f);
                        e[4 * c4] = v4.x; e[4 * c4 + 1] = v4.y; e[4 * c4 + 2] = v4.z; e[4 * c4 + 3] = v4.w;
                    }
#pragma unroll
                    for (int u = 0; u < CHW / 16; ++u) {
                        const int ks = cb * (CHW / 16) + u;
#pragma unroll
                        for (int hs = 0; hs < 2; ++hs) {
                            const float v0 = e[KMap::kdim(ks, 2 * hs, t) - cb * CHW - CH * t];
                            const float v1 = e[KMap::kdim(ks, 2 * hs + 1, t) - cb * CHW - CH * t];
                            const uint32_t hp = P::pack(v0, v1);
                            const float h0 = P::unpack_lo(hp), h1 = P::unpack_lo(hp >> 16);
                            qf[0][nt][ks][hs] = hp;
                            qf[NQ - 1][nt][ks][hs] = P::pack(v0 - h0, v1 - h1);
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
            m_run[nt][0] = m_run[nt][1] = -INFINITY;
            l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
            for (int mi = 0; mi < MT; ++mi)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[nt][mi][e] = 0.f;
        }
        cur_len = seg_len(p, b);
    };

    volatile int* merge_flag = reinterpret_cast<volatile int*>(smem + L::FLAG_OFF + 4);
    // Merge of row z (runs in the CTA whose arrival completed z): obuf and
    // mlbuf are free again here.  Partial of CTA c lives at unit max(zb, ub(c)).
    auto merge = [&](int z, int zb, int c0, int c1) {
        // Runs in the CTA whose arrival completed row z (usually at the very end
        // of the kernel, so its latency is the kernel's tail): every partial
        // statistic is fetched with independent loads into shared memory, then
        // each output element reads all partials at once.
        constexpr int KCH = 32;                  // slots handled through smem
        const int rows = p.rows;
        const int nsl = c1 - c0 + 1;
        float* Mr = mlbuf;            // [16] row max
        float* Lr = mlbuf + 16;       // [16] 1 / row sum
        float* Fw = mlbuf + 32;       // [16] weight of the FP partial
        float* sw = obuf;             // [KCH][16] slot max -> weight
        float* sl_ = obuf + KCH * 16; // [KCH][16] slot sum
        auto slot_of = [&](int j) {
            const int ucc = (int)((int64_t)(c0 + j) * U / C);
            return ucc > zb ? ucc : zb;
        };
        const bool fast = nsl <= KCH;
        if (fast) {
            for (int idx = ctid; idx < nsl * rows; idx += kConsumerWarps * 32) {
                const int j = idx / rows, r = idx % rows;
                const float2 ml = *reinterpret_cast<const float2*>(p.ws_ml + ((int64_t)slot_of(j) * rows + r) * 2);
                sw[j * 16 + r] = ml.x;
                sl_[j * 16 + r] = ml.y;
            }
            named_bar_sync(1, kConsumerWarps * 32);
        }
        if (ctid < rows) {
            const int r = ctid;
            const float2 fml = p.fp_ml ? *reinterpret_cast<const float2*>(p.fp_ml + ((int64_t)z * rows + r) * 2)
                                       : make_float2(-INFINITY, 0.f);
            float M = fml.x;
            for (int j = 0; j < nsl; ++j)
                M = fmaxf(M, fast ? sw[j * 16 + r] : p.ws_ml[((int64_t)slot_of(j) * rows + r) * 2]);
            const float fw = (fml.x == -INFINITY) ? 0.f : ex2(fml.x - M);
            float Ls = fw * fml.y;
            for (int j = 0; j < nsl; ++j) {
                const float ms = fast ? sw[j * 16 + r] : p.ws_ml[((int64_t)slot_of(j) * rows + r) * 2];
                const float ls = fast ? sl_[j * 16 + r] : p.ws_ml[((int64_t)slot_of(j) * rows + r) * 2 + 1];
                const float w = (ms == -INFINITY) ? 0.f : ex2(ms - M);
                Ls += w * ls;
                if (fast) sw[j * 16 + r] = w;
            }
            Mr[r] = M;
            Lr[r] = Ls > 0.f ? 1.f / Ls : 0.f;
            Fw[r] = fw;
        }
        named_bar_sync(1, kConsumerWarps * 32);
        constexpr int PER = NT * 8 * D / (kConsumerWarps * 32);   // outputs per thread (upper bound)
        float acc[PER];
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int i = ctid + k * kConsumerWarps * 32;
            acc[k] = 0.f;
            if (i >= rows * D) continue;
            const int r = i / D;
            if (fast) {
#pragma unroll 8
                for (int j = 0; j < nsl; ++j) {
                    const float w = sw[j * 16 + r];
                    if (w != 0.f) acc[k] = fmaf(w, p.ws_o[(int64_t)slot_of(j) * rows * D + i], acc[k]);
                }
            } else {
                for (int j = 0; j < nsl; ++j) {
                    const float ms = p.ws_ml[((int64_t)slot_of(j) * rows + r) * 2];
                    if (ms != -INFINITY) acc[k] = fmaf(ex2(ms - Mr[r]), p.ws_o[(int64_t)slot_of(j) * rows * D + i], acc[k]);
                }
            }
        }
        named_bar_sync(1, kConsumerWarps * 32);
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int i = ctid + k * kConsumerWarps * 32;
            if (i < rows * D) obuf[i] = acc[k];
        }
        named_bar_sync(1, kConsumerWarps * 32);
        const int b = z / p.Hkv, h = z % p.Hkv;
        auto* out = reinterpret_cast<typename Elem<DT>::T*>(p.out);
        for (int i = ctid; i < rows * D; i += kConsumerWarps * 32) {
            const int r = i / D, d = i % D;
            float mid = obuf[i];
            if (p.rotation) {
                mid = 0.f;
                for (int e = 0; e < D; ++e) mid = fmaf(obuf[r * D + e], p.rotation[(int64_t)e * D + d], mid);
            }
            float v = mid;
            if (p.fp_o) v = fmaf(Fw[r], p.fp_o[(int64_t)z * rows * D + i], v);
            v *= Lr[r];
            const int j = r / p.n_q, sq = r % p.n_q;
            out[(int64_t)b * p.o_sb + (int64_t)(h * p.g + j) * p.o_sh + (int64_t)sq * p.o_ss + d] = Elem<DT>::from_f(v);
        }
    };

    auto flush = [&](int z) {
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
        if (gid == 0) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int r = nt * 8 + 2 * t + e;
                    mlbuf[(warp * 16 + r) * 2 + 0] = m_run[nt][e];
                    mlbuf[(warp * 16 + r) * 2 + 1] = l_run[nt][e];
                }
        }
        named_bar_sync(1, kConsumerWarps * 32);
        // 2) rescale this warp's O to the CTA max and accumulate into obuf
        float f[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int r = nt * 8 + 2 * t + e;
                float M = -INFINITY;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mlbuf[(w * 16 + r) * 2]);
                f[nt][e] = (m_run[nt][e] == -INFINITY) ? 0.f : ex2(m_run[nt][e] - M);
            }
        for (int pass = 0; pass < kConsumerWarps; ++pass) {
            if (warp == pass) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int mi = 0; mi < MT; ++mi)
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int r = nt * 8 + 2 * t + (e & 1);
                            const int d = VMap::vdim(mi, e >> 1, gid);
                            const float v = o[nt][mi][e] * f[nt][e & 1];
                            if (pass == 0) obuf[r * D + d] = v; else obuf[r * D + d] += v;
                        }
            }
            named_bar_sync(1, kConsumerWarps * 32);
        }
        // 3) write the CTA partial for z to its slot: the first unit of z this
        //    CTA processed (unique per CTA, inside z's unit range)
        const int zb = units_begin(p, z);
        const int slot = zb > ub ? zb : ub;
        float* go = p.ws_o + (int64_t)slot * p.rows * D;
        for (int i = ctid; i < p.rows * D; i += kConsumerWarps * 32) go[i] = obuf[i];
        if (ctid < p.rows) {
            const int r = ctid;
            float M = -INFINITY, Ls = 0.f;
            for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mlbuf[(w * 16 + r) * 2]);
            for (int w = 0; w < kConsumerWarps; ++w) {
                const float mw = mlbuf[(w * 16 + r) * 2];
                if (mw != -INFINITY) Ls += ex2(mw - M) * mlbuf[(w * 16 + r) * 2 + 1];
            }
            p.ws_ml[((int64_t)slot * p.rows + r) * 2 + 0] = M;
            p.ws_ml[((int64_t)slot * p.rows + r) * 2 + 1] = Ls;
        }
        // 4) count the arrival; the last CTA of row z merges every partial of
        //    z (FP tiers + one per middle CTA) and writes the output.  No CTA
        //    ever waits for another: the merge runs where the count completes.
        __threadfence();
        named_bar_sync(1, kConsumerWarps * 32);
        const int ze = units_begin(p, z + 1);
        const int c0 = cta_of_unit(zb, C, U), c1 = cta_of_unit(ze - 1, C, U);
        if (ctid == 0) {
            const int old = atomicAdd(p.counters + z, 1);
            *merge_flag = (old == c1 - c0) ? 1 : 0;
        }
        named_bar_sync(1, kConsumerWarps * 32);
        if (*merge_flag) {
            __threadfence();
            FADE_TR(38);
            merge(z, zb, c0, c1);
            FADE_TR(39);
        }
        named_bar_sync(1, kConsumerWarps * 32);
    };

    int z = z_of_unit(p, Z, ub);
    int zb = units_begin(p, z), ze = units_begin(p, z + 1);

    for (int u = ub, i = 0; u < ue; ++u, ++i) {
        while (u >= ze) { ++z; zb = ze; ze = units_begin(p, z + 1); }
        if (z != cur_z) {
            if (FADE_ABLATE != 6) {
                FADE_TR(2 + 3 * (cur_z >= 0 ? 1 : 0));
                if (cur_z >= 0) flush(cur_z);
                FADE_TR(3 + 3 * (cur_z >= 0 ? 1 : 0));
                setup_z(z);
                FADE_TR(4 + 3 * (cur_z >= 0 ? 1 : 0));
            }
            cur_z = z;
        }
        const int s = i % kStages;
        const uint32_t ph = (uint32_t)(i / kStages) & 1u;
        const bool ready = mbar_wait(full_bar(s), ph, abort_flag, p.ws_err);
        FADE_TR(10 + i);
        const int64_t tok_w = (int64_t)(u - zb) * kStageTokens + warp * 32;  // first token of this warp
        const uint8_t* st = smem + s * L::STAGE_BYTES;
        const uint32_t kbase = smem_u32(st + L::K_OFF);
        const uint32_t vbase = smem_u32(st + L::V_OFF);
        const uint8_t* scb = smem + L::SC_BASE + s * L::SC_BYTES;

        if (ready && tok_w < cur_len && FADE_ABLATE != 1 && FADE_ABLATE < 4) {
            // ---- S^T = K_deq . q^T for the warp's 2 m-tiles ----
            // two accumulators per m-tile (even / odd k-steps) halve the
            // dependent MMA chain; summed before the softmax
            float sacc[2][NT][4], sacc2[2][NT][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) sacc[mt][nt][e] = sacc2[mt][nt][e] = 0.f;
                uint32_t kr[2][L::NCHK];
                load_tiles<L::NCHK, false>(kbase, warp * 32 + mt * 16, lane, kr);
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
                                    P::mma((ks & 1) ? sacc2[mt][nt] : sacc[mt][nt], a0, a1, a2, a3,
                                           qf[qs][nt][ks][0], qf[qs][nt][ks][1]);
                        }
                    } else {
                        uint32_t h0[8], h1[8];
                        Conv<DT>::int2(kr[0][cb], h0);
                        Conv<DT>::int2(kr[1][cb], h1);
#pragma unroll
                        for (int u4 = 0; u4 < 4; ++u4) {
                            const int ks = cb * 4 + u4;
                            const uint32_t a0 = P::mul(h0[2 * u4], ksc[ks][0]);
                            const uint32_t a1 = P::mul(h1[2 * u4], ksc[ks][0]);
                            const uint32_t a2 = P::mul(h0[2 * u4 + 1], ksc[ks][1]);
                            const uint32_t a3 = P::mul(h1[2 * u4 + 1], ksc[ks][1]);
#pragma unroll
                            for (int qs = 0; qs < NQ; ++qs)
#pragma unroll
                                for (int nt = 0; nt < NT; ++nt)
                                    P::mma((ks & 1) ? sacc2[mt][nt] : sacc[mt][nt], a0, a1, a2, a3,
                                           qf[qs][nt][ks][0], qf[qs][nt][ks][1]);
                        }
                    }
                }
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) sacc[mt][nt][e] += sacc2[mt][nt][e];
            // ---- online softmax over the 32 tokens (log2 domain) ----
            uint32_t pb[2][NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int tok = (int)tok_w + mt * 16 + gid + ((e >> 1) << 3);
                        float v = sacc[mt][nt][e] * p.qk_scale;
                        if (tok >= cur_len) v = -INFINITY;
                        sacc[mt][nt][e] = v;
                        mx[e & 1] = fmaxf(mx[e & 1], v);
                    }
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 4));
                    mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 8));
                    mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], 16));
                    const float mnew = fmaxf(m_run[nt][e], mx[e]);
                    const float corr = (m_run[nt][e] == -INFINITY) ? 0.f : ex2(m_run[nt][e] - mnew);
                    m_run[nt][e] = mnew;
                    l_run[nt][e] *= corr;
#pragma unroll
                    for (int mi = 0; mi < MT; ++mi) {
                        o[nt][mi][e] *= corr;
                        o[nt][mi][e + 2] *= corr;
                    }
                }
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    float pv[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float mref = m_run[nt][e & 1];
                        const float pe = (sacc[mt][nt][e] == -INFINITY) ? 0.f : ex2(sacc[mt][nt][e] - mref);
                        l_run[nt][e & 1] += pe;
                        pv[e] = pe;
                    }
                    pb[mt][nt][0] = movmatrix_t(P::pack(pv[0], pv[1]));
                    pb[mt][nt][1] = movmatrix_t(P::pack(pv[2], pv[3]));
                }
            }
            // ---- O^T += V_deq^T . P^T ----
#pragma unroll
            for (int mt = 0; mt < (FADE_ABLATE == 2 ? 0 : 2); ++mt) {
                const int trow0 = warp * 32 + mt * 16;
                uint32_t vr[2][L::NCHV];
                load_tiles<L::NCHV, true>(vbase, trow0, lane, vr);
                // tokens of this m-tile past the length: their scales may be
                // stale bytes (NaN * 0 must not reach the MMA), so zero them;
                // a tile entirely past the length is skipped.
                const int64_t tile_tok = tok_w - warp * 32 + trow0;
                if (tile_tok >= cur_len) continue;
                uint32_t vs0 = 0, vs1 = 0;
                const uint16_t* gsc = nullptr;
                if constexpr (!VGROUP) {
                    const uint32_t* sc32 = reinterpret_cast<const uint32_t*>(scb);
                    vs0 = sc32[(trow0 + 2 * t) >> 1];       // tokens 2t, 2t+1
                    vs1 = sc32[(trow0 + 8 + 2 * t) >> 1];   // tokens 8+2t, 9+2t
                    const int64_t rem = cur_len - tile_tok;  // valid tokens in this tile (> 0)
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
                        Conv<DT>::int2(vr[0][cb], h0);
                        Conv<DT>::int2(vr[1][cb], h1);
                        // channels +0 h[3], +1 h[2], +2 h[1], +3 h[0], +4 h[7], +5 h[6], +6 h[5], +7 h[4]
                        const int lo[4] = {3, 1, 7, 5};
                        const int hi[4] = {2, 0, 6, 4};
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int mi = cb * 4 + j;
                            uint32_t a0, a1, a2, a3;
                            if constexpr (!VGROUP) {
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
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(s));
    }
    FADE_TR(36);
    if (cur_z >= 0 && FADE_ABLATE != 6) flush(cur_z);
    FADE_TR(37);
}

// ---------------------------------------------------------------------------
// k0: q_rot = q @ R^T (fp32), one CTA per query row
// ---------------------------------------------------------------------------
template <int DT>
__global__ void rotate_queries_kernel(const void* q, int Hq, int n_q, int D, int64_t q_sb,
                                      int64_t q_sh, int64_t q_ss, const float* __restrict__ R,
                                      float* __restrict__ q_rot) {
    griddep_wait();
    griddep_launch_dependents();
    extern __shared__ float qs[];
    const int row = blockIdx.x;  // (b*Hq + hq)*n_q + s
    const int s = row % n_q, bh = row / n_q;
    const int hq = bh % Hq, b = bh / Hq;
    const int64_t off = (int64_t)b * q_sb + (int64_t)hq * q_sh + (int64_t)s * q_ss;
    for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = load_f<DT>(q, off + d);
    __syncthreads();
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float acc = 0.f;
        for (int e = 0; e < D; ++e) acc = __fadd_rn(acc, __fmul_rn(qs[e], R[(int64_t)d * D + e]));
        q_rot[(int64_t)row * D + d] = acc;
    }
}

// ---------------------------------------------------------------------------
// k_fp: attention over the FP (model-dtype) tiers -- sinks and the recent
// window -- one CTA per (b, kv-head).  With a quantised middle it writes an
// un-normalised partial (m, l, O) that the middle kernel's merge consumes;
// otherwise (or for a row with no middle units) it writes the final output.
// Lanes of a warp take 8 tokens x 4 channel quarters for q.k (16-byte loads)
// and own D/32 channels each for p.v (coalesced rows).
// ---------------------------------------------------------------------------
struct FpSeg {
    const void* k;
    const void* v;
    int64_t row_sb, row_sh;
    const int64_t* row_base;
    const int32_t* lens;
    int64_t len;
};
struct FpParams {
    int B, Hq, Hkv, D, n_q, g, rows;
    float qk_scale;
    const void* q;
    int64_t q_sb, q_sh, q_ss;
    void* out;
    int64_t o_sb, o_sh, o_ss;
    int n_fp;
    FpSeg fp[FADE_MAX_SEGMENTS];
    int has_mid;
    const int32_t* cu_units;        // middle units per row (ragged) or null
    int units_per_z;
    float* ws_fpml;                 // [Z][rows][2]
    float* ws_fpo;                  // [Z][rows][D]
    int* counters;                  // [Z] middle-kernel arrival counters (zeroed here)
    int vec;                        // FP rows 16-byte aligned: vector loads
};

template <int DT, int N>
__device__ __forceinline__ void load_row_part(const typename Elem<DT>::T* src, bool vec, bool valid,
                                              float (&dst)[N]) {
    if (!valid) {
#pragma unroll
        for (int e = 0; e < N; ++e) dst[e] = 0.f;
        return;
    }
    if constexpr (N % 8 == 0) {
        if (vec) {
#pragma unroll
            for (int c = 0; c < N / 8; ++c) {
                const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src) + c);
                const auto* e8 = reinterpret_cast<const typename Elem<DT>::T*>(&raw);
#pragma unroll
                for (int e = 0; e < 8; ++e) dst[c * 8 + e] = Elem<DT>::to_f(e8[e]);
            }
            return;
        }
    }
#pragma unroll
    for (int e = 0; e < N; ++e) dst[e] = Elem<DT>::to_f(src[e]);
}

template <int DT, int D, int NT>
__global__ void __launch_bounds__(kFpThreads)
fp_tier_kernel(FpParams p) {
    constexpr int ROWS = NT * 8;
    constexpr int DPL = D / 32;      // channels per lane in p.v
    constexpr int DQ = D / 4;        // channels per lane in q.k
    constexpr int QS = DQ + 4;       // padded quarter stride: quarters hit different banks
    constexpr int RS = 4 * QS;
    constexpr int NW = kFpThreads / 32;
    griddep_wait();
    griddep_launch_dependents();
    __shared__ __align__(16) float qsm[ROWS * RS];
    __shared__ float osm[ROWS * D];
    __shared__ float msm[NW][ROWS], lsm[NW][ROWS];
    __shared__ float fin_m[ROWS], fin_l[ROWS];

    const int z = blockIdx.x;
    const int b = z / p.Hkv, h = z % p.Hkv;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int rows = p.rows;
    // The middle kernel (next in the stream, started only after this grid
    // completes) counts arrivals per row here; start every call from zero.
    if (threadIdx.x == 0 && p.counters) p.counters[z] = 0;

    for (int i = threadIdx.x; i < ROWS * D; i += kFpThreads) {
        const int r = i / D, d = i % D;
        float v = 0.f;
        if (r < rows) {
            const int j = r / p.n_q, sq = r % p.n_q;
            v = load_f<DT>(p.q, (int64_t)b * p.q_sb + (int64_t)(h * p.g + j) * p.q_sh + (int64_t)sq * p.q_ss + d) *
                p.qk_scale;
        }
        qsm[r * RS + (d / DQ) * QS + d % DQ] = v;
        osm[i] = 0.f;
    }
    __syncthreads();

    float m[ROWS], l[ROWS], o[ROWS][DPL];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        m[r] = -INFINITY;
        l[r] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[r][e] = 0.f;
    }
    const int tk = lane >> 2, qd = lane & 3;
    for (int si = 0; si < p.n_fp; ++si) {
        const FpSeg& sg = p.fp[si];
        const int64_t len = sg.lens ? (int64_t)sg.lens[b] : sg.len;
        const int64_t row0 = sg.row_base ? sg.row_base[z] : (int64_t)b * sg.row_sb + (int64_t)h * sg.row_sh;
        const auto* K = reinterpret_cast<const typename Elem<DT>::T*>(sg.k);
        const auto* V = reinterpret_cast<const typename Elem<DT>::T*>(sg.v);
        for (int64_t t0 = (int64_t)warp * 8; t0 < len; t0 += (int64_t)NW * 8) {
            const int64_t tok = t0 + tk;
            const bool tv = tok < len;
            float kd[DQ];
            load_row_part<DT, DQ>(K + (row0 + (tv ? tok : 0)) * D + qd * DQ, p.vec != 0, tv, kd);
            // the group's 8 V rows are requested together with K (one latency)
            float vv[8][DPL];
#pragma unroll
            for (int tt = 0; tt < 8; ++tt) {
                const int64_t tk2 = t0 + tt;
                const auto* vr = V + (row0 + (tk2 < len ? tk2 : 0)) * D + lane * DPL;
#pragma unroll
                for (int e = 0; e < DPL; ++e) vv[tt][e] = tk2 < len ? Elem<DT>::to_f(vr[e]) : 0.f;
            }
            float sc[ROWS];
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
                const float4* qv = reinterpret_cast<const float4*>(qsm + r * RS + qd * QS);
                float acc = 0.f;
#pragma unroll
                for (int e4 = 0; e4 < DQ / 4; ++e4) {
                    const float4 q4 = qv[e4];
                    acc = fmaf(q4.x, kd[4 * e4], acc);
                    acc = fmaf(q4.y, kd[4 * e4 + 1], acc);
                    acc = fmaf(q4.z, kd[4 * e4 + 2], acc);
                    acc = fmaf(q4.w, kd[4 * e4 + 3], acc);
                }
                acc += __shfl_xor_sync(0xffffffffu, acc, 1);
                acc += __shfl_xor_sync(0xffffffffu, acc, 2);
                sc[r] = tv ? acc : -INFINITY;
            }
            float pr[ROWS];
#pragma unroll
            for (int r = 0; r < ROWS; ++r) {
                float mx = sc[r];
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                const float mnew = fmaxf(m[r], mx);
                const float corr = (m[r] == -INFINITY) ? 0.f : ex2(m[r] - mnew);
                m[r] = mnew;
                pr[r] = (sc[r] == -INFINITY) ? 0.f : ex2(sc[r] - mnew);
                float ps = (qd == 0) ? pr[r] : 0.f;
                ps += __shfl_xor_sync(0xffffffffu, ps, 4);
                ps += __shfl_xor_sync(0xffffffffu, ps, 8);
                ps += __shfl_xor_sync(0xffffffffu, ps, 16);
                l[r] = l[r] * corr + ps;
#pragma unroll
                for (int e = 0; e < DPL; ++e) o[r][e] *= corr;
            }
#pragma unroll
            for (int tt = 0; tt < 8; ++tt) {
#pragma unroll
                for (int r = 0; r < ROWS; ++r) {
                    const float pt = __shfl_sync(0xffffffffu, pr[r], tt * 4);
#pragma unroll
                    for (int e = 0; e < DPL; ++e) o[r][e] = fmaf(pt, vv[tt][e], o[r][e]);
                }
            }
        }
    }
    if (lane == 0) {
#pragma unroll
        for (int r = 0; r < ROWS; ++r) { msm[warp][r] = m[r]; lsm[warp][r] = l[r]; }
    }
    __syncthreads();
    if (threadIdx.x < ROWS) {
        const int r = threadIdx.x;
        float M = -INFINITY, Ls = 0.f;
        for (int w = 0; w < NW; ++w) M = fmaxf(M, msm[w][r]);
        for (int w = 0; w < NW; ++w)
            if (msm[w][r] != -INFINITY) Ls += ex2(msm[w][r] - M) * lsm[w][r];
        fin_m[r] = M;
        fin_l[r] = Ls;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const float f = (m[r] == -INFINITY) ? 0.f : ex2(m[r] - fin_m[r]);
#pragma unroll
        for (int e = 0; e < DPL; ++e) atomicAdd(&osm[r * D + lane * DPL + e], o[r][e] * f);
    }
    __syncthreads();
    int units_z = 0;
    if (p.has_mid) units_z = p.cu_units ? p.cu_units[z + 1] - p.cu_units[z] : p.units_per_z;
    if (units_z > 0) {
        for (int i = threadIdx.x; i < rows * D; i += kFpThreads) p.ws_fpo[(int64_t)z * rows * D + i] = osm[i];
        if (threadIdx.x < rows) {
            p.ws_fpml[((int64_t)z * rows + threadIdx.x) * 2 + 0] = fin_m[threadIdx.x];
            p.ws_fpml[((int64_t)z * rows + threadIdx.x) * 2 + 1] = fin_l[threadIdx.x];
        }
    } else {
        auto* out = reinterpret_cast<typename Elem<DT>::T*>(p.out);
        for (int i = threadIdx.x; i < rows * D; i += kFpThreads) {
            const int r = i / D, d = i % D;
            const int j = r / p.n_q, sq = r % p.n_q;
            const float v = fin_l[r] > 0.f ? osm[i] / fin_l[r] : 0.f;
            out[(int64_t)b * p.o_sb + (int64_t)(h * p.g + j) * p.o_sh + (int64_t)sq * p.o_ss + d] = Elem<DT>::from_f(v);
        }
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
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, &middle_kernel<DT, D, KB, VB, VG, NT, QS>,
                                                      kMidThreads, i.smem);
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
    return MidKernelInfo{nullptr, 0, 0};
}

template <int DT>
static MidKernelInfo select_mid_d(int D, int NT, int kb, int vb, bool vg, bool rot) {
    if (D == 128) return NT == 1 ? select_mid<DT, 128, 1>(kb, vb, vg, rot) : select_mid<DT, 128, 2>(kb, vb, vg, rot);
    if (D == 64) return NT == 1 ? select_mid<DT, 64, 1>(kb, vb, vg, rot) : select_mid<DT, 64, 2>(kb, vb, vg, rot);
    return MidKernelInfo{nullptr, 0, 0};
}

template <int DT>
static void* select_fp(int D, int NT) {
    if (D == 128) return NT == 1 ? (void*)&fp_tier_kernel<DT, 128, 1> : (void*)&fp_tier_kernel<DT, 128, 2>;
    if (D == 64) return NT == 1 ? (void*)&fp_tier_kernel<DT, 64, 1> : (void*)&fp_tier_kernel<DT, 64, 2>;
    return nullptr;
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
    size_t off_err, off_qrot, off_cnt, off_fpml, off_fpo, off_ml, off_o, total;
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
        } else return FADE_ERR_INVALID_ARG;
        if (!s.k || !s.v || !s.k_scale || !s.v_scale) return FADE_ERR_INVALID_ARG;
        if (!aligned16(s.k) || !aligned16(s.v)) return FADE_ERR_ALIGN;
        if (s.lens && s.max_len <= 0 && !d->cu_units) return FADE_ERR_INVALID_ARG;
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
    pl->off_cnt = off; off += ((size_t)Z * 4 + 255) / 256 * 256;
    pl->off_fpml = off; off += ((size_t)Z * pl->rows * 2 * 4 + 255) / 256 * 256;
    pl->off_fpo = off; off += ((size_t)Z * pl->rows * d->D * 4 + 255) / 256 * 256;
    pl->off_ml = off; off += ((size_t)pl->max_units * pl->rows * 2 * 4 + 255) / 256 * 256;
    pl->off_o = off; off += (size_t)pl->max_units * pl->rows * d->D * 4;
    pl->total = off;
    return FADE_OK;
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

extern "C" int fade_decode_attn(const fade_decode_desc* d, void* workspace, size_t ws_bytes,
                                void* stream) {
    Plan pl;
    int st = make_plan(d, &pl);
    if (st != FADE_OK) return st;
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
        void* fn = d->dtype == FADE_F16 ? (void*)&rotate_queries_kernel<FADE_F16>
                                        : (void*)&rotate_queries_kernel<FADE_BF16>;
        const void* qp = d->q;
        int Hq = d->Hq, nq = d->n_q, D = d->D;
        int64_t a = d->q_sb, b2 = d->q_sh, c2 = d->q_ss;
        const float* R = d->rotation;
        void* args[] = {(void*)&qp, &Hq, &nq, &D, &a, &b2, &c2, (void*)&R, (void*)&qrot};
        FADE_CUDA_TRY(launch_pdl(fn, dim3((unsigned)(d->B * d->Hq * d->n_q)), dim3(128),
                                 (size_t)d->D * 4, s, args));
    }
    // FP tiers: a partial for the merge, or the final output when there is no
    // middle (and for ragged rows whose middle is empty).
    // Always launched: with a middle tier it also zeroes the arrival counters
    // (the workspace may have held another call's partials there).
    const bool run_fp = true;
    if (run_fp) {
        FpParams fp = {};
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
        fp.has_mid = has_mid ? 1 : 0;
        fp.cu_units = d->cu_units;
        fp.units_per_z = pl.units_per_z;
        fp.ws_fpml = reinterpret_cast<float*>(ws + pl.off_fpml);
        fp.ws_fpo = reinterpret_cast<float*>(ws + pl.off_fpo);
        fp.counters = has_mid ? reinterpret_cast<int*>(ws + pl.off_cnt) : nullptr;
        void* fn = d->dtype == FADE_F16 ? select_fp<FADE_F16>(d->D, pl.NT) : select_fp<FADE_BF16>(d->D, pl.NT);
        if (!fn) return FADE_ERR_UNSUPPORTED;
        void* args[] = {(void*)&fp};
        FADE_CUDA_TRY(launch_pdl(fn, dim3((unsigned)Z), dim3(kFpThreads), 0, s, args));
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
            if (sg.row_base) return FADE_ERR_INVALID_ARG;
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
        mp.units_per_z = pl.units_per_z;
        mp.n_ctas = pl.n_ctas;
        mp.ws_ml = reinterpret_cast<float*>(ws + pl.off_ml);
        mp.ws_o = reinterpret_cast<float*>(ws + pl.off_o);
        mp.ws_err = reinterpret_cast<int*>(ws + pl.off_err);
        mp.counters = reinterpret_cast<int*>(ws + pl.off_cnt);
        mp.fp_ml = pl.n_fp > 0 ? reinterpret_cast<const float*>(ws + pl.off_fpml) : nullptr;
        mp.fp_o = pl.n_fp > 0 ? reinterpret_cast<const float*>(ws + pl.off_fpo) : nullptr;
        mp.out = d->out; mp.o_sb = d->o_sb; mp.o_sh = d->o_sh; mp.o_ss = d->o_ss;
        mp.rotation = rot ? d->rotation : nullptr;
        mp.scale_tma = scale_tma;
        if (std::getenv("FADE_DEBUG_PLAN")) {
            std::fprintf(stderr,
                         "[fade] decode plan: B=%d Hq=%d Hkv=%d D=%d rows=%d kb=%d vb=%d grouped=%d "
                         "units/z=%d ctas=%d occ=%d smem=%d scale_tma=%d n_rows=%lld\n",
                         d->B, d->Hq, d->Hkv, d->D, pl.rows, pl.kb, pl.vb, (int)pl.vg, pl.units_per_z,
                         pl.n_ctas, pl.mk.occ, pl.mk.smem, scale_tma, (long long)n_rows);
        }
        mp.q_vec = aligned16(sg.k_scale) && sg.ks_sb % 8 == 0 && sg.ks_sh % 8 == 0 &&
                   (rot || (aligned16(d->q) && d->q_sb % 8 == 0 && d->q_sh % 8 == 0 && d->q_ss % 8 == 0));
        void* args[] = {(void*)&tk, (void*)&tv, (void*)&ts, (void*)&mp};
        FADE_CUDA_TRY(launch_pdl(pl.mk.fn, dim3((unsigned)pl.n_ctas), dim3(kMidThreads),
                                 (size_t)pl.mk.smem, s, args));
    }
    return FADE_OK;
}

extern "C" int fade_workspace_check(void* workspace, size_t ws_bytes, void* stream) {
    if (!workspace || ws_bytes < 256) return FADE_ERR_WORKSPACE;
    int h = 0;
    cudaStream_t s = as_stream(stream);
    FADE_CUDA_TRY(cudaMemcpyAsync(&h, workspace, sizeof(int), cudaMemcpyDeviceToHost, s));
    FADE_CUDA_TRY(cudaStreamSynchronize(s));
    if (h != 0) {
        // A stalled call may have left arrival counters mid-count: zero it all.
        FADE_CUDA_TRY(cudaMemsetAsync(workspace, 0, ws_bytes, s));
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
    // The array keeps the previous call's bytes.  Only the error word must
    // start at zero (the per-row arrival counters are reset by the call's own
    // FP-tier kernel), so clear the first 256 bytes on the caller's stream.
    FADE_CUDA_TRY(cudaMemsetAsync(ws, 0, 256, as_stream(stream)));
    return fade_decode_attn(d, ws, fade::kNoAllocScratchBytes, stream);
}

#ifdef FADE_TRACE
extern "C" int fade_trace_read(unsigned long long* host, size_t n) {
    const size_t bytes = n * sizeof(unsigned long long) < sizeof(fade::g_trace) ? n * sizeof(unsigned long long)
                                                                               : sizeof(fade::g_trace);
    return cudaMemcpyFromSymbol(host, fade::g_trace, bytes) == cudaSuccess ? 0 : 7;
}
extern "C" int fade_trace_clear(void) {
    static unsigned long long zeros[1024 * fade::kTraceEv];
    return cudaMemcpyToSymbol(fade::g_trace, zeros, sizeof(zeros)) == cudaSuccess ? 0 : 7;
}
#endif
