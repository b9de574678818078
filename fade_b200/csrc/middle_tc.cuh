// Tensor-core (tcgen05) middle kernel: INT4 K and V, D = 128, up to 16
// query rows per kv head.  Included by decode.cu after the mma.sync middle
// kernel, whose helpers (mbarriers, TMA, code conversion, FP-tier warp, unit
// schedule) it shares; it writes the same partials (one per CTA and row, at
// the first unit of the row it processed), so the same finisher merges them
// (with one "group" per CTA).
//
// Per 128-token stage of a (b, kv-head) row:
//   * the TMA producer warp streams K and V codes and V scales into a ring;
//   * a dequantisation warpgroup (two of them, alternating stages) turns the
//     codes into exact model-dtype values rnd(c * s) (as fade/quant.py:124-127)
//     and writes K into tensor memory (lane = token, 2 channels per 32-bit
//     column: the A operand of S^T = K q^T) and V into shared memory (token
//     rows, 128B-swizzled: the MN-major A operand of O^T = V^T P^T);
//   * one thread issues tcgen05.mma: S^T[128 x 16] into TMEM, later
//     O^T[128 channels x 16] += V^T P^T into TMEM, and commits each to an
//     mbarrier;
//   * the softmax warpgroup reads S^T from TMEM (lane = token), keeps running
//     maxima (log2 domain; kept while new scores stay within 2^8 of them, else
//     O is rescaled in TMEM), writes P^T in the model dtype to shared memory
//     (K-major B operand) and, at the row's last stage, reads O^T and stores
//     the CTA's partial (max, sum, un-normalised O).
// Channels appear inside the MMAs in the order the code conversion produces
// them: K index (and V^T row) 8m + p holds channel 8m + kTcPerm[p]; the query
// tile is written in the same order and O^T is un-permuted at the store.
// Register use per thread stays small (no MMA fragments or accumulators in
// registers).  Selected with fade_set_middle_kernel(1); the mma.sync kernel
// stays the default because it is faster on B200: here every 128-token stage
// passes a chain of hand-offs (conversion -> QK MMA -> softmax -> PV MMA ->
// buffer release), each a few hundred nanoseconds of mbarrier / tcgen05
// commit / tensor-memory load latency, and with two stage buffers that chain,
// not the conversion's instruction count, sets the time per stage.

constexpr int kTcNS = 6;            // ring stages (16 KB of codes each)
constexpr int kTcN = 16;            // MMA N: query rows, zero-padded
constexpr int kTcThreads = 512;
constexpr int kTcCols = 256;        // TMEM columns allocated
constexpr int kTcColK = 0;          // K tiles: 2 x 64 columns
constexpr int kTcColS = 128;        // S^T: 2 x 16 columns
constexpr int kTcColO = 160;        // O^T: 16 columns

// K index p (within 8) -> channel offset, the order Conv<DT>::int4 emits
// (h[0] = (e1, e5), h[1] = (e0, e4), h[2] = (e3, e7), h[3] = (e2, e6))
__host__ __device__ constexpr int kTcPerm(int p) {
    return p == 0 ? 1 : p == 1 ? 5 : p == 2 ? 0 : p == 3 ? 4 : p == 4 ? 3 : p == 5 ? 7 : p == 6 ? 2 : 6;
}

struct TcLayout {
    static constexpr int K_BYTES = kStageTokens * 64;
    static constexpr int STAGE = 2 * K_BYTES;                    // K codes, V codes
    static constexpr int RING_OFF = 0;
    static constexpr int SC_OFF = kTcNS * STAGE;                 // per-stage V scales
    static constexpr int SC_BYTES = kStageTokens * 2;
    static constexpr int VB_OFF = ((SC_OFF + kTcNS * SC_BYTES + 1023) / 1024) * 1024;
    static constexpr int VB_BYTES = kStageTokens * 128 * 2;      // dequantised V, 32 KB
    static constexpr int Q_OFF = VB_OFF + 2 * VB_BYTES;
    static constexpr int QP_BYTES = kTcN * 128 * 2;              // 4 KB
    static constexpr int P_OFF = Q_OFF + 2 * QP_BYTES;
    static constexpr int KS_OFF = P_OFF + 2 * QP_BYTES;          // K scale pairs, per warpgroup
    static constexpr int KS_BYTES = 64 * 4;
    static constexpr int RED_OFF = KS_OFF + 2 * KS_BYTES;        // softmax reductions [2][4][16]
    static constexpr int BAR_OFF = RED_OFF + 2 * 4 * kTcN * 4;
    static constexpr int N_BARS = 2 * kTcNS + 12;
    static constexpr int TSLOT_OFF = BAR_OFF + N_BARS * 8;
    static constexpr int FLAG_OFF = TSLOT_OFF + 8;
    static constexpr int AB_OFF = ((FLAG_OFF + 8 + 15) / 16) * 16;
    static constexpr int AB_BYTES = 2 * kFpChunk * (128 + 8) * 2;
    static constexpr int SMEM_BYTES = AB_OFF + AB_BYTES + 1024;  // +1024 for alignment
    static_assert(SMEM_BYTES <= kSmemPerBlock, "tcgen05 middle kernel shared memory over the per-CTA limit");
    static_assert(VB_OFF % 1024 == 0 && (Q_OFF % 1024) == 0, "128B-swizzled operands need 1 KB alignment");
};

// Bounded wait for the pipeline hand-offs of this kernel: polls with plain
// try_wait (which returns as soon as the phase completes) rather than the
// suspend-hint form, whose sleeps add microseconds to every hand-off of a
// pipeline whose stages wait on each other.  Gives up after kTcPolls polls
// (the CTA then aborts and reports through the error word).
constexpr uint32_t kTcPolls = 1u << 22;
__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
    for (uint32_t i = 0; i < kTcPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && *abort_flag) return false;
    }
    *abort_flag = 1;
    atomicExch(err, 1);
    return false;
}

// Instruction descriptor, kind::f16: f32 accumulator, A and B in the model
// dtype, M = 128, N = kTcN; a_mn: A is MN-major.
template <int DT>
__host__ __device__ constexpr uint32_t tc_idesc(bool a_mn) {
    return (1u << 4) | ((DT == FADE_BF16 ? 1u : 0u) << 7) | ((DT == FADE_BF16 ? 1u : 0u) << 10) |
           ((a_mn ? 1u : 0u) << 15) | ((uint32_t)(kTcN >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
// K-major, no swizzle: element (row n, k) of a [16 x 128] operand tile
__device__ __forceinline__ uint32_t tc_kmajor_off(int n, int k) {
    return (uint32_t)((n >> 3) * 2048 + (k >> 3) * 128 + (n & 7) * 16 + (k & 7) * 2);
}

template <int DT, int NT>
__global__ void __launch_bounds__(kTcThreads, 1)
    middle_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                     const __grid_constant__ CUtensorMap tmap_s, const MidParams p) {
    constexpr int D = 128;
    using L = TcLayout;
    using P = Pk<DT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sb = smem_u32(smem);
    // shared-memory accesses by 32-bit shared address, as ordinary loads and
    // stores through the shared pointer (ordered by the compiler against the
    // barrier and tcgen05 asm, which clobber memory)
    auto sp = [&](uint32_t addr) { return smem + (addr - sb); };
    auto lds128 = [&](uint32_t addr) { return *reinterpret_cast<const uint4*>(sp(addr)); };
    auto sts128 = [&](uint32_t addr, uint4 v) { *reinterpret_cast<uint4*>(sp(addr)) = v; };
    auto sts32 = [&](uint32_t addr, uint32_t v) { *reinterpret_cast<uint32_t*>(sp(addr)) = v; };
    auto sts16 = [&](uint32_t addr, uint16_t v) { *reinterpret_cast<uint16_t*>(sp(addr)) = v; };
    const uint32_t bar0 = sb + L::BAR_OFF;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kTcNS + s); };
    const uint32_t b1 = bar0 + 8u * (2 * kTcNS);
    auto kv_full = [&](int b) { return b1 + 8u * b; };
    auto kv_free = [&](int b) { return b1 + 8u * (2 + b); };
    auto s_full = [&](int b) { return b1 + 8u * (4 + b); };
    auto s_free = [&](int b) { return b1 + 8u * (6 + b); };
    auto p_full = [&](int b) { return b1 + 8u * (8 + b); };
    const uint32_t fin_bar = b1 + 8u * 10;   // every MMA of the CTA complete
    const uint32_t o_free = b1 + 8u * 11;    // a row's partial read out of O^T

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int Z = p.B * p.Hkv;
    const int U = total_units(p, Z);
    const int C = p.n_ctas < U ? p.n_ctas : U;
    const int c = blockIdx.x;
    const bool streams = c < C;
    const int ub = streams ? (int)((int64_t)c * U / C) : 0;
    const int ue = streams ? (int)((int64_t)(c + 1) * U / C) : 0;
    const int n = ue - ub;   // stages of this CTA
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::FLAG_OFF);

    if (threadIdx.x == 0) {
        *abort_flag = 0;
        for (int s = 0; s < kTcNS; ++s) {
            mbar_init(full_bar(s), 32);
            mbar_init(empty_bar(s), 128);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(kv_full(b), 128);
            mbar_init(kv_free(b), 1);
            mbar_init(s_full(b), 1);
            mbar_init(s_free(b), 128);
            mbar_init(p_full(b), 128);
        }
        mbar_init(fin_bar, 1);
        mbar_init(o_free, 128);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // zero the query and P tiles once: rows past p.rows stay zero
    for (int i = threadIdx.x; i < 4 * L::QP_BYTES / 16; i += blockDim.x)
        sts128(sb + L::Q_OFF + 16u * i, make_uint4(0u, 0u, 0u, 0u));
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (warp == 1 && n > 0) {
        tc_alloc(sb + L::TSLOT_OFF, kTcCols);
        tc_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = n > 0 ? *reinterpret_cast<volatile uint32_t*>(smem + L::TSLOT_OFF) : 0u;

    const bool fp_early = p.early && warp == 2;
    if (!(p.early && warp == 0) && !fp_early) griddep_wait();
    if (warp >= 4) griddep_launch_dependents();
    if (warp == 2) {
        fp_rows_warp_body<DT, D, NT>(p, c, (int)gridDim.x, smem + L::AB_OFF, !fp_early);
        return;
    }
    if (warp == 3 || n <= 0) return;

    if (warp == 0) {
        // ------------------------------ producer ------------------------------
        const uint64_t policy = evict_first_policy();
        if (lane == 0) {
            prefetch_tmap(&tmap_k);
            prefetch_tmap(&tmap_v);
            if (p.scale_tma) prefetch_tmap(&tmap_s);
        }
        int z = z_of_unit(p, Z, ub);
        int zb = units_begin(p, z), ze = units_begin(p, z + 1);
        int64_t zrow0 = seg_row0(p, z), zlen = seg_len(p, z / p.Hkv);
        for (int i = 0; i < n; ++i) {
            const int s = i % kTcNS;
            const uint32_t ph = (uint32_t)(i / kTcNS) & 1u;
            const int u = ub + i;
            if (u >= ze) {
                while (u >= ze) { ++z; zb = ze; ze = units_begin(p, z + 1); }
                zrow0 = seg_row0(p, z);
                zlen = seg_len(p, z / p.Hkv);
            }
            if (!tc_wait(empty_bar(s), ph ^ 1u, abort_flag, p.ws_err)) continue;
            const int64_t tok0 = (int64_t)(u - zb) * kStageTokens;
            const int64_t row0 = p.page_table
                ? (int64_t)__ldg(p.page_table + (int64_t)z * p.pages_per_row + (u - zb)) * kStageTokens
                : zrow0 + tok0;
            const uint32_t st = sb + L::RING_OFF + s * L::STAGE;
            const uint32_t scs = sb + L::SC_OFF + s * L::SC_BYTES;
            if (lane == 0 && tok0 < zlen) {
                mbar_expect_tx(full_bar(s), (uint32_t)L::STAGE + (p.scale_tma ? (uint32_t)L::SC_BYTES : 0u));
                tma_load_2d(st, &tmap_k, 0, (int)(row0 * 64 / 128), full_bar(s), policy);
                tma_load_2d(st + L::K_BYTES, &tmap_v, 0, (int)(row0 * 64 / 128), full_bar(s), policy);
                if (p.scale_tma) tma_load_1d(scs, &tmap_s, (int)row0, full_bar(s), policy);
            }
            if (!p.scale_tma && tok0 < zlen) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int tt = lane * 4 + j;
                    sts16(scs + 2u * tt, (tok0 + tt < zlen) ? load_bits<DT>(p.v_scale, row0 + tt) : (uint16_t)0);
                }
            }
            mbar_arrive(full_bar(s));
        }
        // drain: every ring slot released, so no TMA write lands after exit
        for (int i = n; i < n + kTcNS; ++i) {
            if (i - kTcNS < 0) continue;
            tc_wait(empty_bar(i % kTcNS), ((uint32_t)(i / kTcNS) & 1u) ^ 1u, abort_flag, p.ws_err);
        }
        return;
    }

    // stage -> row bookkeeping shared by the roles below
    struct RowWalk {
        int z, zb, ze;
    };
    auto walk_init = [&](RowWalk& w) {
        w.z = z_of_unit(p, Z, ub);
        w.zb = units_begin(p, w.z);
        w.ze = units_begin(p, w.z + 1);
    };
    auto walk_to = [&](RowWalk& w, int u) {
        while (u >= w.ze) { ++w.z; w.zb = w.ze; w.ze = units_begin(p, w.z + 1); }
    };

    if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        {
            // the whole warp polls (uniform results); one elected lane issues
            constexpr uint32_t IQK = tc_idesc<DT>(false), IPV = tc_idesc<DT>(true);
            RowWalk w;
            walk_init(w);
            int row_idx = -1;   // rows started by this CTA so far - 1
            // Two in-order streams, each issued as soon as its inputs are
            // ready (non-blocking polls): QK(i) once stage i is converted and
            // S^T buffer i % 2 was read; PV(j) once P(j) is written.  PV(j)
            // never waits behind QK(j + 1), so the conversion of stage j + 2
            // (which waits for PV(j)) overlaps the conversion of stage j + 1.
            int nq = 0, np = 0;
            uint32_t idle = 0;
            while (np < n) {
                bool did = false;
                if (nq < n) {
                    const int b = nq & 1;
                    if (mbar_test_wait(kv_full(b), (uint32_t)(nq >> 1) & 1u) &&
                        (nq < 2 || mbar_test_wait(s_free(b), (uint32_t)((nq >> 1) - 1) & 1u))) {
                        tc_fence_after();
                        const uint32_t qb = sb + L::Q_OFF + b * L::QP_BYTES;
                        if (elect_one()) {
#pragma unroll
                        for (int ks = 0; ks < D / 16; ++ks)
                            tc_mma_ts(tmem + kTcColS + 16 * b, tmem + kTcColK + 64 * b + 8 * ks,
                                      tc_desc(qb + ks * 256, 128, 2048, 0), IQK, ks > 0 ? 1u : 0u);
                        tc_commit(s_full(b));
                        }
                        __syncwarp();
                        ++nq;
                        did = true;
                    }
                }
                if (np < nq) {
                    const int b = np & 1;
                    const int u = ub + np;
                    walk_to(w, u);
                    const bool first = (np == 0) || (u == w.zb);
                    // a new row also needs the previous row's partial read out of O^T
                    if (mbar_test_wait(p_full(b), (uint32_t)(np >> 1) & 1u) &&
                        (!first || row_idx < 0 || mbar_test_wait(o_free, (uint32_t)row_idx & 1u))) {
                        if (first) ++row_idx;
                        tc_fence_after();
                        const uint32_t vb = sb + L::VB_OFF + b * L::VB_BYTES;
                        const uint32_t pb = sb + L::P_OFF + b * L::QP_BYTES;
                        if (elect_one()) {
#pragma unroll
                        for (int ks = 0; ks < kStageTokens / 16; ++ks)
                            tc_mma_ss(tmem + kTcColO, tc_desc(vb + ks * 2048, L::VB_BYTES / 2, 1024, 2),
                                      tc_desc(pb + ks * 256, 128, 2048, 0), IPV, (first && ks == 0) ? 0u : 1u);
                        tc_commit(kv_free(b));
                        }
                        __syncwarp();
                        ++np;
                        did = true;
                    }
                }
                if (did) {
                    idle = 0;
                } else {
                    ++idle;
                    if ((idle & 255u) == 0u && *abort_flag) break;
                    if (idle > kTcPolls * 8u) {
                        *abort_flag = 1;
                        atomicExch(p.ws_err, 1);
                        break;
                    }
                }
            }
            // every MMA of the CTA complete before TMEM is released
            if (elect_one()) tc_commit(fin_bar);
            __syncwarp();
            tc_wait(fin_bar, 0u, abort_flag, p.ws_err);
        }
        __syncwarp();
        named_bar_sync(4, 13 * 32);   // MMA warp + both conversion groups + softmax group
        tc_fence_after();
        tc_dealloc(tmem, kTcCols);
        return;
    }

    const int grp = (warp - 4) / 4;   // 0: conversion group 0, 1: softmax, 2: conversion group 1
    const int tl = threadIdx.x % 128; // TMEM lane / token (conversion, softmax) or channel (O^T)
    const uint32_t lane_base = (uint32_t)(32 * (warp % 4)) << 16;

    if (grp != 1) {
        // --------------------------- conversion groups ---------------------------
        const int d = grp == 0 ? 0 : 1;
        const int bar_id = 1 + d;
        const uint32_t ksb = sb + L::KS_OFF + d * L::KS_BYTES;
        const uint32_t qb = sb + L::Q_OFF + d * L::QP_BYTES;
        const uint32_t vb = sb + L::VB_OFF + d * L::VB_BYTES;
        RowWalk w;
        walk_init(w);
        int cur_z = -1;
        int64_t cur_len = 0;
        for (int i = d; i < n; i += 2) {
            const int s = i % kTcNS;
            const int u = ub + i;
            walk_to(w, u);
            // buffers of stage i - 2 (K tile, V tile, query tile) free again
            bool ok = (i < 2) || tc_wait(kv_free(d), (uint32_t)((i >> 1) - 1) & 1u, abort_flag, p.ws_err);
            if (w.z != cur_z) {
                // new row: K scale pairs in conversion order, query tile
                named_bar_sync(bar_id, 128);   // everyone done with the previous row's scales
                const int b = w.z / p.Hkv, h = w.z % p.Hkv;
                const int64_t ks_off = (int64_t)b * p.ks_sb + (int64_t)h * p.ks_sh;
                if (tl < 64) {
                    const int m = tl >> 2, i2 = tl & 3;
                    const uint16_t lo = load_bits<DT>(p.k_scale, ks_off + 8 * m + kTcPerm(2 * i2));
                    const uint16_t hi = load_bits<DT>(p.k_scale, ks_off + 8 * m + kTcPerm(2 * i2 + 1));
                    sts32(ksb + 4u * tl, (uint32_t)lo | ((uint32_t)hi << 16));
                }
                {
                    const int k = tl, ch = 8 * (k >> 3) + kTcPerm(k & 7);
                    for (int r = 0; r < p.rows; ++r) {
                        const int j = r / p.n_q, sq = r % p.n_q;
                        const int64_t qoff = (int64_t)b * p.q_sb + (int64_t)(h * p.g + j) * p.q_sh +
                                             (int64_t)sq * p.q_ss;
                        sts16(qb + tc_kmajor_off(r, k), load_bits<DT>(p.q, qoff + ch));
                    }
                }
                cur_z = w.z;
                cur_len = seg_len(p, b);
                named_bar_sync(bar_id, 128);
            }
            ok = ok && tc_wait(full_bar(s), (uint32_t)(i / kTcNS) & 1u, abort_flag, p.ws_err);
            if (ok) {
                const bool valid = (int64_t)(u - w.zb) * kStageTokens + tl < cur_len;
                const uint32_t st = sb + L::RING_OFF + s * L::STAGE;
                const int R = tl >> 1, half = tl & 1;
                // ---- K: rnd(c * s_channel) into TMEM, lane tl ----
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const uint4 wv = lds128(st + R * 128 + (((half * 4 + j4) ^ (R & 7)) * 16));
                    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
                    uint32_t out[16];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint32_t hh[4];
                        Conv<DT>::int4(wd[q], hh);
                        const uint4 sc = lds128(ksb + (4 * j4 + q) * 16);
                        out[4 * q + 0] = P::mul(hh[0], sc.x);
                        out[4 * q + 1] = P::mul(hh[1], sc.y);
                        out[4 * q + 2] = P::mul(hh[2], sc.z);
                        out[4 * q + 3] = P::mul(hh[3], sc.w);
                    }
                    tc_st16(tmem + lane_base + kTcColK + 64 * d + 16 * j4, out);
                }
                // ---- V: rnd(c * s_token) into the 128B-swizzled token rows ----
                const uint16_t vsb = *reinterpret_cast<const uint16_t*>(smem + L::SC_OFF + s * L::SC_BYTES + 2 * tl);
                const uint32_t vs2 = valid ? dup16(vsb) : 0u;
                const uint32_t vrow = vb + (tl >> 3) * 1024 + (tl & 7) * 128;
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const uint4 wv = lds128(st + L::K_BYTES + R * 128 + (((half * 4 + j4) ^ (R & 7)) * 16));
                    const uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint32_t hh[4];
                        Conv<DT>::int4(wd[q], hh);
                        const int m = 4 * j4 + q;   // 8-channel word: M half m / 8, chunk m % 8
                        uint4 o4;
                        o4.x = valid ? P::mul(hh[0], vs2) : 0u;
                        o4.y = valid ? P::mul(hh[1], vs2) : 0u;
                        o4.z = valid ? P::mul(hh[2], vs2) : 0u;
                        o4.w = valid ? P::mul(hh[3], vs2) : 0u;
                        sts128(vrow + (m >> 3) * (L::VB_BYTES / 2) + (((m & 7) ^ (tl & 7)) * 16), o4);
                    }
                }
                mbar_arrive(empty_bar(s));
                tc_wait_st();
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                tc_fence_before();
                mbar_arrive(kv_full(d));
            }
        }
    } else {
        // ------------------------------ softmax group ------------------------------
        const float qks = p.qk_scale;
        const int rows = p.rows;
        constexpr int RM = 8 * NT;   // query rows this instantiation serves (rows <= RM)
        float m_run[RM], l_thr[RM];
#pragma unroll
        for (int r = 0; r < RM; ++r) { m_run[r] = kMaskedMax; l_thr[r] = 0.f; }
        float* red = reinterpret_cast<float*>(smem + L::RED_OFF);
        RowWalk w;
        walk_init(w);
        int64_t cur_len = 0;
        int row_idx = -1;
        for (int i = 0; i < n; ++i) {
            const int b = i & 1;
            const int u = ub + i;
            walk_to(w, u);
            const bool first = (i == 0) || (u == w.zb);
            const bool last = (i == n - 1) || (u + 1 == w.ze);
            if (first) {
                ++row_idx;
                cur_len = seg_len(p, w.z / p.Hkv);
#pragma unroll
                for (int r = 0; r < RM; ++r) { m_run[r] = kMaskedMax; l_thr[r] = 0.f; }
            }
            bool ok = tc_wait(s_full(b), (uint32_t)(i >> 1) & 1u, abort_flag, p.ws_err);
            uint32_t sv[16];
            if (ok) {
                tc_fence_after();
                tc_ld16(tmem + lane_base + kTcColS + 16 * b, sv);
            } else {
#pragma unroll
                for (int r = 0; r < 16; ++r) sv[r] = 0u;
            }
            tc_fence_before();
            mbar_arrive(s_free(b));
            const bool valid = (int64_t)(u - w.zb) * kStageTokens + tl < cur_len;
            float x[RM];
#pragma unroll
            for (int r = 0; r < RM; ++r) x[r] = (valid && r < rows) ? __uint_as_float(sv[r]) * qks : -INFINITY;
            // block maxima over the 128 tokens
            float* rb = red + (i & 1) * (4 * kTcN);
#pragma unroll
            for (int r = 0; r < RM; ++r) {
                if (r < rows) {
                    float v = x[r];
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
                    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
                    if (lane == 0) rb[(warp % 4) * kTcN + r] = v;
                }
            }
            named_bar_sync(3, 128);
            bool grow = false;
            float bm[RM];
#pragma unroll
            for (int r = 0; r < RM; ++r) {
                bm[r] = kMaskedMax;
                if (r < rows) {
                    bm[r] = fmaxf(fmaxf(rb[r], rb[kTcN + r]), fmaxf(rb[2 * kTcN + r], rb[3 * kTcN + r]));
                    bm[r] = fmaxf(bm[r], kMaskedMax);
                    grow |= bm[r] > m_run[r] + 8.f;
                }
            }
            // PV(i - 2) complete: P buffer b is free, and (commits complete in
            // issue order) every earlier PV too, so the waits below on the
            // next phases of kv_free are well defined
            if (ok && i >= 2) ok = tc_wait(kv_free(b), (uint32_t)((i >> 1) - 1) & 1u, abort_flag, p.ws_err);
            if (first) {
#pragma unroll
                for (int r = 0; r < RM; ++r) m_run[r] = bm[r];
            } else if (grow) {
                // rescale O^T (lane = channel) once the previous stage's PV is done
                float corr[RM];
#pragma unroll
                for (int r = 0; r < RM; ++r) {
                    const float mn = fmaxf(m_run[r], bm[r]);
                    corr[r] = ex2(m_run[r] - mn);
                    m_run[r] = mn;
                    l_thr[r] *= corr[r];
                }
                if (ok) ok = tc_wait(kv_free((i - 1) & 1), (uint32_t)((i - 1) >> 1) & 1u, abort_flag, p.ws_err);
                if (ok) {
                    tc_fence_after();
                    uint32_t ov[16];
                    tc_ld16(tmem + lane_base + kTcColO, ov);
#pragma unroll
                    for (int r = 0; r < RM; ++r) ov[r] = __float_as_uint(__uint_as_float(ov[r]) * corr[r]);
                    tc_st16(tmem + lane_base + kTcColO, ov);
                    tc_wait_st();
                }
            }
            // P = exp2(x - m) in the model dtype, as the K-major B operand [16 x 128 tokens]
            const uint32_t pb = sb + L::P_OFF + b * L::QP_BYTES;
#pragma unroll
            for (int r = 0; r < RM; ++r) {
                if (r < rows) {
                    const float pe = ex2(x[r] - m_run[r]);
                    l_thr[r] += pe;
                    const uint32_t bits = P::pack(pe, 0.f) & 0xFFFFu;
                    const uint32_t other = __shfl_xor_sync(0xffffffffu, bits, 1);
                    if ((lane & 1) == 0 && ok) sts32(pb + tc_kmajor_off(r, tl), bits | (other << 16));
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            mbar_arrive(p_full(b));
            if (last) {
                // ---- the CTA's partial of this row ----
                if (ok) ok = tc_wait(kv_free(b), (uint32_t)(i >> 1) & 1u, abort_flag, p.ws_err);
                uint32_t ov[16];
                if (ok) {
                    tc_fence_after();
                    tc_ld16(tmem + lane_base + kTcColO, ov);
                }
                tc_fence_before();
                mbar_arrive(o_free);
                // row sums over the 128 tokens
                float lsum[RM];
#pragma unroll
                for (int r = 0; r < RM; ++r) {
                    lsum[r] = 0.f;
                    if (r < rows) {
                        float v = l_thr[r];
                        v += __shfl_xor_sync(0xffffffffu, v, 16);
                        v += __shfl_xor_sync(0xffffffffu, v, 8);
                        v += __shfl_xor_sync(0xffffffffu, v, 4);
                        v += __shfl_xor_sync(0xffffffffu, v, 2);
                        v += __shfl_xor_sync(0xffffffffu, v, 1);
                        lsum[r] = v;
                    }
                }
                // the other reduction buffer is free: the next stage's maxima
                // use buffer (i + 1) & 1 only after the barrier below
                float* lr = red + ((i + 1) & 1) * (4 * kTcN);
                named_bar_sync(3, 128);
                if (lane == 0) {
#pragma unroll
                    for (int r = 0; r < RM; ++r)
                        if (r < rows) lr[(warp % 4) * kTcN + r] = lsum[r];
                }
                named_bar_sync(3, 128);
                const int slot = w.zb > ub ? w.zb : ub;
                if (ok) {
                    const int ch = 8 * (tl >> 3) + kTcPerm(tl & 7);
                    float* go = p.ws_o + (int64_t)slot * rows * D;
#pragma unroll
                    for (int r = 0; r < RM; ++r)
                        if (r < rows) go[r * D + ch] = __uint_as_float(ov[r]);
#pragma unroll
                    for (int r = 0; r < RM; ++r) {
                        if (r < rows && tl == r) {
                            const float Ls = (lr[r] + lr[kTcN + r]) + (lr[2 * kTcN + r] + lr[3 * kTcN + r]);
                            *reinterpret_cast<float2*>(p.ws_ml + ((int64_t)slot * rows + r) * 2) =
                                make_float2(m_run[r], Ls);
                        }
                    }
                }
                named_bar_sync(3, 128);   // lr read before the next stage's maxima reuse it
            }
        }
    }
    named_bar_sync(4, 13 * 32);
}
