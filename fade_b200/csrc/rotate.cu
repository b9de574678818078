// Rotated quantisation (fade/rotated_quant.py): x_rot = x @ R^T in fp32, then
// symmetric quantisation at 2/3/4 bits with fp32 math, K per-channel over S,
// V per-token.  The dot products accumulate e = 0..D-1 sequentially with
// separately rounded products and sums (no FMA contraction), a fixed order the
// CPU oracle restates exactly.  The reference's CPU matmul (MKL) sums in its
// own order, so codes match it except where a rotated value sits within an
// fp32 ulp of a rounding boundary.
#include "common.cuh"
#include "sm100.cuh"

namespace fade {

constexpr int kRotTokens = 64;   // tokens per CTA
constexpr int kRotAcc = 32;      // tokens per thread: independent accumulation chains
constexpr int kRotThreads = 256;

// y[t][d] = sum_e in[t][e] * M[e][d] for the kRotTokens tokens of a tile,
// each output summed in e order with separately rounded products and sums.
// Thread (d, g) computes channel d of kRotTokens / (blockDim.x / D) tokens:
// that many independent chains, inputs read four channels at a time (one
// broadcast 16-byte load).  DC > 0 fixes D at compile time (no predication);
// DC == 0 is the generic form.  `y` may alias `in`: the results are written
// after a block-wide barrier.
template <int DC>
__device__ __forceinline__ void rot_matmul(const float* in, const float* __restrict__ M, int ldm, float* y, int D_rt) {
    const int D = DC > 0 ? DC : D_rt;
    const int groups = blockDim.x / D;                          // >= 2 for D <= 128
    const int tpg = (kRotTokens + groups - 1) / groups;         // <= kRotAcc
    const int d = threadIdx.x % D, t0 = (threadIdx.x / D) * tpg;
    const bool on = threadIdx.x < groups * D;
    const int nj = !on ? 0 : ((kRotTokens - t0) < tpg ? (kRotTokens - t0) : tpg);
    constexpr int NJ = DC > 0 ? kRotTokens / (256 / (DC > 0 ? DC : 1)) : kRotAcc;
    float acc[NJ];
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[j] = 0.f;
    if (on) {
        for (int e = 0; e < D; e += 4) {
            const float m0 = M[e * ldm + d], m1 = M[(e + 1) * ldm + d], m2 = M[(e + 2) * ldm + d],
                        m3 = M[(e + 3) * ldm + d];
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                if (DC > 0 || j < nj) {
                    const float4 x = *reinterpret_cast<const float4*>(in + (t0 + j) * D + e);
                    float a = acc[j];
                    a = __fadd_rn(a, __fmul_rn(x.x, m0));
                    a = __fadd_rn(a, __fmul_rn(x.y, m1));
                    a = __fadd_rn(a, __fmul_rn(x.z, m2));
                    a = __fadd_rn(a, __fmul_rn(x.w, m3));
                    acc[j] = a;
                }
            }
        }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NJ; ++j)
        if (DC > 0 || j < nj) y[(t0 + j) * D + d] = acc[j];
}

__device__ __forceinline__ void qrange(int bits, float& lo, float& hi) {
    lo = (float)(-(1 << (bits - 1)));
    hi = (float)((1 << (bits - 1)) - 1);
}

// Rotate kRotTokens rows of (b,h) into xs (fp32 [kRotTokens][D]; xs may be xin).
template <int DT, int DC>
__device__ void rotate_tile(const typename Elem<DT>::T* __restrict__ x, const fade_view4& v, int64_t b,
                            int64_t h, int64_t t0, int nt, const float* __restrict__ Rt, float* xin,
                            float* xs) {
    const int D = (int)v.D;
    for (int i = threadIdx.x; i < kRotTokens * D; i += blockDim.x) {
        const int t = i / D, e = i % D;
        xin[i] = (t < nt) ? Elem<DT>::to_f(x[b * v.sb + h * v.sh + (t0 + t) * v.ss + (int64_t)e * v.sd]) : 0.f;
    }
    __syncthreads();
    rot_matmul<DC>(xin, Rt, D + 1, xs, D);
    __syncthreads();
}

// pass 0 (K only): per-channel absmax of x_rot into amax (float bits, atomicMax).
// pass 1: quantise.  kind 0 = K (per-channel scale from amax), 1 = V (per-token).
template <int DT, int DC>
__global__ void __launch_bounds__(kRotThreads)
rotated_quant_kernel(const typename Elem<DT>::T* __restrict__ x, fade_view4 v, const float* __restrict__ R,
                     int bits, int kind, int pass, float* __restrict__ amax, uint8_t* __restrict__ packed,
                     typename Elem<DT>::T* __restrict__ scale) {
    extern __shared__ float sm[];
    const int D = (int)v.D;
    float* Rt = sm;                    // [D][D+1] transposed: Rt[e][d] = R[d][e]
    float* xin = Rt + D * (D + 1);     // [kRotTokens][D]
    float* xs = xin;                   // the rotation is written over its input
    float* tsc = xin + kRotTokens * D; // [kRotTokens] per-token inv
    const int64_t tiles = (v.S + kRotTokens - 1) / kRotTokens;
    const int64_t bh = blockIdx.x / tiles, tile = blockIdx.x % tiles;
    const int64_t b = bh / v.H, h = bh % v.H;
    const int64_t t0 = tile * kRotTokens;
    const int nt = (int)min((int64_t)kRotTokens, v.S - t0);
    // R in 16-byte pieces, 8 loads in flight per thread (D % 4 == 0)
#pragma unroll 8
    for (int i = threadIdx.x * 4; i < D * D; i += blockDim.x * 4) {
        const float4 r4 = __ldg(reinterpret_cast<const float4*>(R + i));
        const int d = i / D, e = i % D;
        Rt[e * (D + 1) + d] = r4.x;          // rows padded to D + 1: conflict-free
        Rt[(e + 1) * (D + 1) + d] = r4.y;
        Rt[(e + 2) * (D + 1) + d] = r4.z;
        Rt[(e + 3) * (D + 1) + d] = r4.w;
    }
    __syncthreads();
    rotate_tile<DT, DC>(x, v, b, h, t0, nt, Rt, xin, xs);
    float lo, hi;
    qrange(bits, lo, hi);
    if (kind == 0 && pass == 0) {
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
            float m = 0.f;
            for (int t = 0; t < nt; ++t) m = fmaxf(m, fabsf(xs[t * D + d]));
            atomicMax(reinterpret_cast<int*>(amax) + bh * D + d, __float_as_int(m));
        }
        return;
    }
    if (kind == 1) {
        // per-token absmax over D
        for (int t = threadIdx.x / 32; t < nt; t += blockDim.x / 32) {
            float m = 0.f;
            for (int d = threadIdx.x % 32; d < D; d += 32) m = fmaxf(m, fabsf(xs[t * D + d]));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
            m = fmaxf(m, 1e-8f);
            if (threadIdx.x % 32 == 0) {
                tsc[t] = inv_scale<FADE_F32>(m, hi);
                scale[bh * v.S + t0 + t] = Elem<DT>::from_f(__fdiv_rn(m, hi));
            }
        }
        __syncthreads();
    } else if (tile == 0) {
        for (int d = threadIdx.x; d < D; d += blockDim.x) {
            const float m = fmaxf(amax[bh * D + d], 1e-8f);
            scale[bh * D + d] = Elem<DT>::from_f(__fdiv_rn(m, hi));
        }
    }
    // quantise + pack: one thread per output byte
    const int per_byte = (bits == 4) ? 2 : (bits == 2 ? 4 : 1);
    const int row_bytes = D / per_byte;
    for (int i = threadIdx.x; i < nt * row_bytes; i += blockDim.x) {
        const int t = i / row_bytes, j = i % row_bytes;
        uint32_t byte = 0;
        for (int k = 0; k < per_byte; ++k) {
            const int d = j * per_byte + k;
            const float inv = (kind == 1) ? tsc[t] : inv_scale<FADE_F32>(fmaxf(amax[bh * D + d], 1e-8f), hi);
            const int q = quant_code(__fmul_rn(xs[t * D + d], inv), lo, hi);
            if (bits == 4) byte |= (uint32_t)(q & 15) << (4 - 4 * k);
            else if (bits == 2) byte |= (uint32_t)(q & 3) << (6 - 2 * k);
            else byte = (uint32_t)(q & 255);
        }
        packed[(bh * v.S + t0 + t) * row_bytes + j] = (uint8_t)byte;
    }
}

// ---------------------------------------------------------------------------
// Tensor-core rotation (bf16 inputs, D = 128, 2- and 4-bit codes).
//
// R (fp32) is split into three bf16 parts, R = R0 + R1 + R2 exactly (each part
// the bf16 rounding of what the previous parts leave), so every product
// x_e * Rj[d][e] of a bf16 input is exact in fp32 and x_rot = sum_j x Rj^T is
// the exact dot product up to the fp32 accumulation inside the tensor core
// (as close to the exact value as the fixed sequential order of the CUDA-core
// kernel above, but in another order: the two can differ in the last fp32
// bit, and a code only where a rotated value sits that close to a rounding
// boundary, as against the reference's own matmul).
//
// One CTA per SM, persistent over 128-token tiles of the [B, H, S] row space.
// Shared memory holds the three R parts and three token tiles (cp.async,
// two tiles ahead: tiles i + 1 and i + 2 load while tile i is multiplied and
// quantised, enough bytes in flight per SM to keep HBM busy), all
// in the canonical K-major layout without swizzle (8-row x 16-byte core
// matrices, 128 bytes apart along K, 2048 bytes apart along the rows).  One
// elected thread issues 3 x 8 tcgen05.mma (M = N = 128, K = 16) into one of
// two 128-column fp32 accumulators in tensor memory (tile i + 1's MMAs run
// while tile i is quantised from the other); then warpgroup g reads
// columns [32 g, 32 g + 32) of every token (thread r of the group: token r,
// tcgen05.ld, 16 columns at a time) and quantises them in fp32 exactly like
// the CUDA-core kernel (per-token maxima combined across the four groups in
// shared memory), each thread storing its 32 codes with one vector store.
// ---------------------------------------------------------------------------
constexpr int kRqGroups = 4;                  // epilogue warpgroups, 32 columns each
constexpr int kRqThreads = 128 * kRqGroups;
constexpr int kRqParts = 3;
constexpr uint32_t kRqOp = 128 * 128 * 2;   // one [128 x 128] bf16 operand
constexpr uint32_t kRqR = 0;                                   // R parts
constexpr int kRqBufs = 3;                                     // token tiles in shared memory
constexpr uint32_t kRqX = kRqR + kRqParts * kRqOp;             // token tiles
constexpr uint32_t kRqBar = kRqX + kRqBufs * kRqOp;            // MMA-done mbarriers, one per accumulator
constexpr uint32_t kRqSlot = kRqBar + 16;                      // tensor-memory address
constexpr uint32_t kRqInv = kRqSlot + 16;                      // [128] per-channel 1/scale
constexpr uint32_t kRqRed = kRqInv + 128 * 4;                  // [4][128] per-warp column maxima
constexpr uint32_t kRqSmem = kRqRed + 4 * 128 * 4 + 1024;      // + alignment
constexpr uint32_t kRqPolls = 1u << 24;

// Set by a rotation kernel whose wait for its MMAs gave up (never expected;
// the outputs of that call are then undefined).  Read with
// fade_rotated_quant_check().
__device__ int g_rotq_error;

__device__ __forceinline__ uint32_t rq_off(int row, int k) {
    return (uint32_t)((row >> 3) * 2048 + (k >> 3) * 128 + (row & 7) * 16 + (k & 7) * 2);
}

// kind::f16 instruction descriptor: f32 accumulator, bf16 A and B, both
// K-major, N = 128, M = 128
constexpr uint32_t kRqIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);

__device__ __forceinline__ void rq_cp16(uint32_t dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}

__global__ void __launch_bounds__(kRqThreads, 1)
rotated_quant_tc_kernel(const __nv_bfloat16* __restrict__ x, fade_view4 v, const float* __restrict__ R, int bits,
                        int kind, int pass, float* __restrict__ amax, uint8_t* __restrict__ packed,
                        __nv_bfloat16* __restrict__ scale) {
    extern __shared__ uint8_t rq_raw[];
    uint8_t* sm = rq_raw + ((1024u - (smem_u32(rq_raw) & 1023u)) & 1023u);
    const uint32_t sb = smem_u32(sm);
    const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
    constexpr int D = 128;
    const int64_t S = v.S, Z = v.B * v.H;
    const int64_t tiles_z = (S + 127) / 128, total = Z * tiles_z;
    float* inv_s = reinterpret_cast<float*>(sm + kRqInv);
    float* red = reinterpret_cast<float*>(sm + kRqRed);

    // R parts: Rj[d][e] at part j, K-major over e
    for (int i = tid * 4; i < D * D; i += kRqThreads * 4) {
        const float4 r4 = __ldg(reinterpret_cast<const float4*>(R + i));
        const int d = i / D, e = i % D;
        const float rr[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float rem = rr[c];
#pragma unroll
            for (int j = 0; j < kRqParts; ++j) {
                const __nv_bfloat16 pj = __float2bfloat16_rn(rem);
                rem -= __bfloat162float(pj);   // exact: pj holds rem's leading bits
                *reinterpret_cast<__nv_bfloat16*>(sm + kRqR + j * kRqOp + rq_off(d, e + c)) = pj;
            }
        }
    }
    if (tid == 0) {
        mbar_init(sb + kRqBar, 1);
        mbar_init(sb + kRqBar + 8, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        tc_alloc(sb + kRqSlot, 256);
        tc_relinquish();
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sm + kRqSlot);
    const uint32_t lane_base = (uint32_t)(32 * (warp % 4)) << 16;   // a warp reaches its quarter of the lanes

    float lo, hi;
    qrange(bits, lo, hi);
    // stage tile t into buffer `buf` (rows past S are zero-filled)
    // this thread's 16-byte pieces of a tile: rows tid / 16 + 32 k, piece tid % 16
    constexpr int kPieces = 128 * 16 / kRqThreads;
    const int row0 = tid / 16, kc = tid % 16;
    const uint32_t doff0 = rq_off(row0, kc * 8);   // + k * 4 * 2048 for row0 + 32 k
    auto load_tile = [&](int64_t t, int buf) {
        const int64_t z = t / tiles_z, t0 = (t % tiles_z) * 128;
        const int64_t b = z / v.H, h = z % v.H;
        const __nv_bfloat16* xr = x + b * v.sb + h * v.sh + (t0 + row0) * v.ss + kc * 8;
        const uint32_t dst0 = sb + kRqX + (uint32_t)buf * kRqOp + doff0;
#pragma unroll
        for (int k = 0; k < kPieces; ++k) {
            const int row = row0 + 32 * k;
            const bool ok = t0 + row < S;
            rq_cp16(dst0 + (uint32_t)k * 4u * 2048u, ok ? xr + (int64_t)(32 * k) * v.ss : xr - row0 * v.ss,
                    ok ? 16u : 0u);
        }
    };

    // MMAs of iteration `i` (tile t) into accumulator i % 2, committed to
    // mbarrier i % 2 (its (i / 2)-th phase)
    auto issue_mma = [&](int i) {
        if (warp == 0) {
            tc_fence_after();
            if (elect_one()) {
                const uint32_t xb = sb + kRqX + (uint32_t)(i % kRqBufs) * kRqOp;
#pragma unroll
                for (int j = 0; j < kRqParts; ++j)
#pragma unroll
                    for (int ks = 0; ks < D / 16; ++ks)
                        tc_mma_ss(tmem + 128u * (uint32_t)(i & 1), tc_desc(xb + ks * 256, 128, 2048, 0),
                                  tc_desc(sb + kRqR + j * kRqOp + ks * 256, 128, 2048, 0), kRqIdesc,
                                  (j | ks) ? 1u : 0u);
                tc_commit(sb + kRqBar + 8u * (uint32_t)(i & 1));
            }
            __syncwarp();
        }
    };
    bool failed = false;
    int it = 0, issued = -1;   // last iteration whose MMAs were issued
    const int64_t G = gridDim.x;
    if ((int64_t)blockIdx.x < total) {
        load_tile(blockIdx.x, 0);
        asm volatile("cp.async.commit_group;" ::: "memory");
        if ((int64_t)blockIdx.x + G < total) load_tile(blockIdx.x + G, 1);
        asm volatile("cp.async.commit_group;" ::: "memory");
        asm volatile("cp.async.wait_group 1;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        issue_mma(0);
        issued = 0;
    }
    for (int64_t t = blockIdx.x; t < total; t += G, ++it) {
        // tile it + 1 landed (all groups complete); its buffer and tile it's
        // stay untouched, tile it + 2 goes to the one that held tile it - 1
        asm volatile("cp.async.wait_group 0;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (t + 2 * G < total) load_tile(t + 2 * G, (it + 2) % kRqBufs);
        asm volatile("cp.async.commit_group;" ::: "memory");
        // accumulator (it + 1) % 2 was last read by tile it - 1's epilogue
        if (t + G < total) {
            issue_mma(it + 1);
            issued = it + 1;
        }
        const int64_t z = t / tiles_z, t0 = (t % tiles_z) * 128;
        // per-channel inverse scales of this row (K, quantisation pass)
        if (kind == 0 && pass == 1 && tid < D) {
            const float m = fmaxf(amax[z * D + tid], 1e-8f);
            inv_s[tid] = inv_scale<FADE_F32>(m, hi);
            if (t0 == 0) scale[z * D + tid] = __float2bfloat16_rn(__fdiv_rn(m, hi));
        }
        uint32_t polls = 0;
        bool timed_out = false;
        while (!mbar_try_wait(sb + kRqBar + 8u * (uint32_t)(it & 1), (uint32_t)(it >> 1) & 1u)) {
            if (++polls == kRqPolls) { timed_out = true; break; }
        }
        // one decision for the whole CTA (also: inv_s written)
        if (__syncthreads_or(timed_out)) {
            if (tid == 0) atomicExch(&g_rotq_error, 1);
            failed = true;
            break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + 128u * (uint32_t)(it & 1);
        const int grp = tid / 128;            // columns [32 grp, 32 grp + 32)
        const int r = tid % 128;              // token row of this thread (its TMEM lane)
        const int q4 = warp % 4;              // the warp's quarter of the lanes
        const uint32_t col0 = 32u * grp;
        const bool valid = t0 + r < S;
        if (kind == 0 && pass == 0) {
            // per-channel maxima over the tile's tokens: each warp reduces its
            // 32 tokens for its group's 32 channels with one redux.sync per
            // channel (non-negative floats order like their bit patterns as
            // unsigned integers), lane j keeping channel j; then the 4
            // quarters combine in shared memory
            uint32_t vv[2][16];
            tc_ld16(acc + lane_base + col0, vv[0]);
            tc_ld16(acc + lane_base + col0 + 16, vv[1]);
            uint32_t mine = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const uint32_t a = valid ? (vv[j / 16][j % 16] & 0x7FFFFFFFu) : 0u;
                uint32_t m;
                asm volatile("redux.sync.max.u32 %0, %1, 0xffffffff;" : "=r"(m) : "r"(a));
                mine = lane == j ? m : mine;
            }
            red[q4 * D + col0 + lane] = __uint_as_float(mine);
            __syncthreads();
            if (tid < D) {
                const float m = fmaxf(fmaxf(red[tid], red[D + tid]), fmaxf(red[2 * D + tid], red[3 * D + tid]));
                atomicMax(reinterpret_cast<int*>(amax) + z * D + tid, __float_as_int(m));
            }
        } else {
            uint32_t vv[2][16];
            tc_ld16(acc + lane_base + col0, vv[0]);
            tc_ld16(acc + lane_base + col0 + 16, vv[1]);
            float inv_t = 0.f;
            if (kind == 1) {
                float m = 0.f;
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int j = 0; j < 16; ++j) m = fmaxf(m, fabsf(__uint_as_float(vv[c][j])));
                red[grp * D + r] = m;
                __syncthreads();
                m = fmaxf(fmaxf(red[r], red[D + r]), fmaxf(red[2 * D + r], red[3 * D + r]));
                m = fmaxf(m, 1e-8f);
                inv_t = inv_scale<FADE_F32>(m, hi);
                if (valid && grp == 0) scale[z * S + t0 + r] = __float2bfloat16_rn(__fdiv_rn(m, hi));
            }
            uint32_t words[4];   // this thread's 32 codes: 16 bytes (4-bit) or 8 (2-bit)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                int q[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float inv = kind == 1 ? inv_t : inv_s[col0 + 16 * c + j];
                    q[j] = quant_code(__fmul_rn(__uint_as_float(vv[c][j]), inv), lo, hi);
                }
                if (bits == 4) {
#pragma unroll
                    for (int w = 0; w < 2; ++w) {
                        uint32_t word = 0;
#pragma unroll
                        for (int k = 0; k < 4; ++k)   // byte k: channels 2k (high nibble), 2k + 1
                            word |= (((uint32_t)(q[8 * w + 2 * k] & 15) << 4) | (uint32_t)(q[8 * w + 2 * k + 1] & 15))
                                    << (8 * k);
                        words[2 * c + w] = word;
                    }
                } else {
                    uint32_t word = 0;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {      // byte k: channels 4k .. 4k + 3 at bits 6, 4, 2, 0
                        uint32_t byte = 0;
#pragma unroll
                        for (int f = 0; f < 4; ++f) byte |= (uint32_t)(q[4 * k + f] & 3) << (6 - 2 * f);
                        word |= byte << (8 * k);
                    }
                    words[c] = word;
                }
            }
            if (valid) {
                if (bits == 4)
                    *reinterpret_cast<uint4*>(packed + (z * S + t0 + r) * (int64_t)64 + 16 * grp) =
                        make_uint4(words[0], words[1], words[2], words[3]);
                else
                    *reinterpret_cast<uint2*>(packed + (z * S + t0 + r) * (int64_t)32 + 8 * grp) =
                        make_uint2(words[0], words[1]);
            }
        }
        tc_fence_before();
        __syncthreads();   // tensor memory read (and red / inv_s) before the next tile's MMAs
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (failed && warp == 0 && issued >= 0) {
        // MMAs may still be in flight: wait (bounded) for the last commit
        // before the tensor memory is released
        const uint32_t bar = sb + kRqBar + 8u * (uint32_t)(issued & 1), par = (uint32_t)(issued >> 1) & 1u;
        for (uint32_t i = 0; i < kRqPolls && !mbar_try_wait(bar, par); ++i) {
        }
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tc_dealloc(tmem, 256);
    }
}

__device__ __forceinline__ int unpack_code(const uint8_t* __restrict__ p, int bits, int64_t row, int D, int d) {
    if (bits == 4) {
        const uint32_t byte = p[row * (D / 2) + d / 2];
        const uint32_t u = (d & 1) ? (byte & 15u) : (byte >> 4);
        return (int)(u & 7u) - (int)(u & 8u);
    }
    if (bits == 2) {
        const uint32_t byte = p[row * (D / 4) + d / 4];
        const uint32_t u = (byte >> (6 - 2 * (d & 3))) & 3u;
        return (int)(u & 1u) - (int)(u & 2u);
    }
    return (int)reinterpret_cast<const int8_t*>(p)[row * D + d];
}

// out = rnd_dt( sum_e rnd_dt(q*scale)[e] * R[e][d] )
template <int DT, int DC>
__global__ void __launch_bounds__(kRotThreads)
rotated_dequant_kernel(const uint8_t* __restrict__ packed, int bits, const typename Elem<DT>::T* __restrict__ scale,
                       int scale_mode, const float* __restrict__ R, int64_t H, int64_t S, int D,
                       typename Elem<DT>::T* __restrict__ out) {
    extern __shared__ float sm[];
    float* Rs = sm;               // [D][D] as given (row e, col d)
    float* xs = Rs + D * D;       // [kRotTokens][D]
    const int64_t tiles = (S + kRotTokens - 1) / kRotTokens;
    const int64_t bh = blockIdx.x / tiles, tile = blockIdx.x % tiles;
    const int64_t t0 = tile * kRotTokens;
    const int nt = (int)min((int64_t)kRotTokens, S - t0);
#pragma unroll 8
    for (int i = threadIdx.x * 4; i < D * D; i += blockDim.x * 4)
        *reinterpret_cast<float4*>(Rs + i) = __ldg(reinterpret_cast<const float4*>(R + i));
    for (int i = threadIdx.x; i < kRotTokens * D; i += blockDim.x) {
        const int t = i / D, e = i % D;
        float val = 0.f;
        if (t < nt) {
            const int64_t row = bh * S + t0 + t;
            const float sc = Elem<DT>::to_f(scale_mode == 0 ? scale[bh * D + e] : scale[row]);
            val = Elem<DT>::rnd(__fmul_rn((float)unpack_code(packed, bits, row, D, e), sc));
        }
        xs[i] = val;
    }
    __syncthreads();
    rot_matmul<DC>(xs, Rs, D, xs, D);
    __syncthreads();
    for (int i = threadIdx.x; i < nt * D; i += blockDim.x)
        out[(bh * S + t0) * D + i] = Elem<DT>::from_f(xs[i]);
}

}  // namespace fade

using namespace fade;

namespace fade {

template <int DT, int DC>
static int launch_rotated_quant(const void* x, fade_view4 xv, const float* R, int bits, int kind, float* amax,
                                size_t need, uint8_t* packed, void* scale, size_t smem, unsigned grid,
                                cudaStream_t st) {
    using T = typename Elem<DT>::T;
    auto k = rotated_quant_kernel<DT, DC>;
    FADE_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    if (kind == 0) {   // pass 0: per-channel absmax of the rotated values
        FADE_CUDA_TRY(cudaMemsetAsync(amax, 0, need, st));
        k<<<grid, kRotThreads, smem, st>>>((const T*)x, xv, R, bits, kind, 0, amax, packed, (T*)scale);
        FADE_LAUNCH_CHECK();
    }
    k<<<grid, kRotThreads, smem, st>>>((const T*)x, xv, R, bits, kind, 1, amax, packed, (T*)scale);
    FADE_LAUNCH_CHECK();
    return FADE_OK;
}

template <int DT>
static int rotated_quant_d(int D, const void* x, fade_view4 xv, const float* R, int bits, int kind, float* amax,
                           size_t need, uint8_t* packed, void* scale, size_t smem, unsigned grid, cudaStream_t st) {
    if (D == 128) return launch_rotated_quant<DT, 128>(x, xv, R, bits, kind, amax, need, packed, scale, smem, grid, st);
    if (D == 64) return launch_rotated_quant<DT, 64>(x, xv, R, bits, kind, amax, need, packed, scale, smem, grid, st);
    return launch_rotated_quant<DT, 0>(x, xv, R, bits, kind, amax, need, packed, scale, smem, grid, st);
}

template <int DT, int DC>
static int launch_rotated_dequant(const uint8_t* packed, int bits, const void* scale, int scale_mode,
                                  const float* R, int64_t H, int64_t S, int D, void* out, size_t smem,
                                  unsigned grid, cudaStream_t st) {
    using T = typename Elem<DT>::T;
    auto k = rotated_dequant_kernel<DT, DC>;
    FADE_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<grid, kRotThreads, smem, st>>>(packed, bits, (const T*)scale, scale_mode, R, H, S, D, (T*)out);
    FADE_LAUNCH_CHECK();
    return FADE_OK;
}

template <int DT>
static int rotated_dequant_d(const uint8_t* packed, int bits, const void* scale, int scale_mode, const float* R,
                             int64_t H, int64_t S, int D, void* out, size_t smem, unsigned grid, cudaStream_t st) {
    if (D == 128)
        return launch_rotated_dequant<DT, 128>(packed, bits, scale, scale_mode, R, H, S, D, out, smem, grid, st);
    if (D == 64)
        return launch_rotated_dequant<DT, 64>(packed, bits, scale, scale_mode, R, H, S, D, out, smem, grid, st);
    return launch_rotated_dequant<DT, 0>(packed, bits, scale, scale_mode, R, H, S, D, out, smem, grid, st);
}

}  // namespace fade

extern "C" int fade_rotated_quant(const void* x, int dtype, fade_view4 xv, const float* R, int bits,
                                  int kind, uint8_t* packed, void* scale, void* workspace,
                                  size_t ws_bytes, void* stream) {
    if (xv.B < 0 || xv.H < 0 || xv.S < 0 || xv.D <= 0) return FADE_ERR_INVALID_ARG;
    if (bits != 2 && bits != 3 && bits != 4) return FADE_ERR_INVALID_ARG;
    if (kind != 0 && kind != 1) return FADE_ERR_INVALID_ARG;
    if ((bits == 4 && xv.D % 2) || (bits == 2 && xv.D % 4)) return FADE_ERR_ODD_DIM;
    if (xv.D > 128 || xv.D % 4) return FADE_ERR_UNSUPPORTED;
    const int64_t Z = xv.B * xv.H;
    if (Z == 0 || xv.S == 0) return FADE_OK;
    if (!x || !R || !packed || !scale) return FADE_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(R) % 16) return FADE_ERR_ALIGN;   // staged with 16-byte loads
    const size_t need = (size_t)Z * xv.D * 4;
    if (kind == 0 && (!workspace || ws_bytes < need)) return FADE_ERR_WORKSPACE;
    cudaStream_t st = as_stream(stream);
    // bf16 at D = 128 with 2- or 4-bit codes and 16-byte rows: tensor cores
    if (dtype == FADE_BF16 && xv.D == 128 && bits != 3 && xv.sd == 1 && aligned16(x) && aligned16(packed) &&
        (xv.sb * 2) % 16 == 0 && (xv.sh * 2) % 16 == 0 && (xv.ss * 2) % 16 == 0) {
        int dev = 0, n_sm = 0;
        FADE_CUDA_TRY(cudaGetDevice(&dev));
        FADE_CUDA_TRY(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
        FADE_CUDA_TRY(cudaFuncSetAttribute(rotated_quant_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kRqSmem));
        const int64_t tiles = Z * ((xv.S + 127) / 128);
        const unsigned g = (unsigned)(tiles < n_sm ? tiles : n_sm);
        float* am = reinterpret_cast<float*>(workspace);
        const auto* xb = reinterpret_cast<const __nv_bfloat16*>(x);
        auto* sc = reinterpret_cast<__nv_bfloat16*>(scale);
        if (kind == 0) {
            FADE_CUDA_TRY(cudaMemsetAsync(am, 0, need, st));
            rotated_quant_tc_kernel<<<g, kRqThreads, kRqSmem, st>>>(xb, xv, R, bits, 0, 0, am, packed, sc);
            FADE_LAUNCH_CHECK();
        }
        rotated_quant_tc_kernel<<<g, kRqThreads, kRqSmem, st>>>(xb, xv, R, bits, kind, 1, am, packed, sc);
        FADE_LAUNCH_CHECK();
        return FADE_OK;
    }
    const int D = (int)xv.D;
    // R (transposed) + one token tile, rotated in place + per-token scales
    const size_t smem = ((size_t)D * (D + 1) + kRotTokens * D + kRotTokens) * 4;
    const int64_t tiles = (xv.S + kRotTokens - 1) / kRotTokens;
    const unsigned grid = (unsigned)(Z * tiles);
    float* amax = reinterpret_cast<float*>(workspace);
    switch (dtype) {
        case FADE_F16: return rotated_quant_d<FADE_F16>(D, x, xv, R, bits, kind, amax, need, packed, scale, smem, grid, st);
        case FADE_BF16: return rotated_quant_d<FADE_BF16>(D, x, xv, R, bits, kind, amax, need, packed, scale, smem, grid, st);
        case FADE_F32: return rotated_quant_d<FADE_F32>(D, x, xv, R, bits, kind, amax, need, packed, scale, smem, grid, st);
        default: return FADE_ERR_INVALID_ARG;
    }
}

extern "C" int fade_rotated_dequant(const uint8_t* packed, int bits, const void* scale, int scale_mode,
                                    const float* R, int dtype, int64_t B, int64_t H, int64_t S, int64_t D,
                                    void* out, void* stream) {
    if (B < 0 || H < 0 || S < 0 || D <= 0) return FADE_ERR_INVALID_ARG;
    if (bits != 2 && bits != 3 && bits != 4) return FADE_ERR_INVALID_ARG;
    if (scale_mode != 0 && scale_mode != 1) return FADE_ERR_INVALID_ARG;
    if (D > 128 || D % 4) return FADE_ERR_UNSUPPORTED;
    const int64_t Z = B * H;
    if (Z == 0 || S == 0) return FADE_OK;
    if (!packed || !scale || !R || !out) return FADE_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(R) % 16) return FADE_ERR_ALIGN;   // staged with 16-byte loads
    const size_t smem = ((size_t)D * D + kRotTokens * D) * 4;   // R + one tile, rotated in place
    const int64_t tiles = (S + kRotTokens - 1) / kRotTokens;
    const unsigned grid = (unsigned)(Z * tiles);
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case FADE_F16: return rotated_dequant_d<FADE_F16>(packed, bits, scale, scale_mode, R, H, S, (int)D, out, smem, grid, st);
        case FADE_BF16: return rotated_dequant_d<FADE_BF16>(packed, bits, scale, scale_mode, R, H, S, (int)D, out, smem, grid, st);
        case FADE_F32: return rotated_dequant_d<FADE_F32>(packed, bits, scale, scale_mode, R, H, S, (int)D, out, smem, grid, st);
        default: return FADE_ERR_INVALID_ARG;
    }
}

extern "C" int fade_rotated_quant_check(void* stream) {
    cudaStream_t st = as_stream(stream);
    int h = 0;
    FADE_CUDA_TRY(cudaMemcpyFromSymbolAsync(&h, g_rotq_error, sizeof(int), 0, cudaMemcpyDeviceToHost, st));
    FADE_CUDA_TRY(cudaStreamSynchronize(st));
    if (h) {
        const int zero = 0;
        FADE_CUDA_TRY(cudaMemcpyToSymbolAsync(g_rotq_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st));
        FADE_CUDA_TRY(cudaStreamSynchronize(st));
        return FADE_ERR_TIMEOUT;
    }
    return FADE_OK;
}
