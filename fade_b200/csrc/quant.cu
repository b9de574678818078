// K1: symmetric quantisation + bit packing kernels, bit-exact with the
// reference's torch arithmetic (fade/quant.py).  These run on tier
// reassignment (per-layer, over the whole middle tier) and on age-out (one
// token per (b, h) per decode step).
//
// Layout rules shared by every kernel here:
//   * INT4 byte d of a row holds codes 2d (high nibble) and 2d+1 (low nibble),
//     two's complement (fade/quant.py:26-43).
//   * 2-bit byte j holds codes 4j..4j+3 at bit offsets 6,4,2,0
//     (fade/rotated_quant.py:35-48).
//   * A thread owns 8 consecutive channels of one token row when D % 8 == 0
//     (one 16-byte load for 16-bit types), else 2 channels.

#include "common.cuh"

namespace fade {

// ---------------------------------------------------------------------------
// Strided element access
// ---------------------------------------------------------------------------
template <int DT, int E>
__device__ __forceinline__ void load_elems(const typename Elem<DT>::T* base, int64_t sd,
                                           bool vec, float (&out)[E]) {
    using T = typename Elem<DT>::T;
    if constexpr (E == 8 && DT != FADE_F32) {
        if (vec) {
            uint4 raw = __ldg(reinterpret_cast<const uint4*>(base));
            const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
            for (int i = 0; i < 8; ++i) out[i] = Elem<DT>::to_f(e[i]);
            return;
        }
    }
#pragma unroll
    for (int i = 0; i < E; ++i) out[i] = Elem<DT>::to_f(base[i * sd]);
}

__device__ __forceinline__ uint32_t pack_nibbles(int hi, int lo) {
    return ((uint32_t)(hi & 0xF) << 4) | (uint32_t)(lo & 0xF);
}

__device__ __forceinline__ uint32_t pack_crumbs(int c0, int c1, int c2, int c3) {
    return ((uint32_t)(c0 & 3) << 6) | ((uint32_t)(c1 & 3) << 4) | ((uint32_t)(c2 & 3) << 2) |
           (uint32_t)(c3 & 3);
}

// Write E/2 packed INT4 bytes for E codes.
template <int E>
__device__ __forceinline__ void store_int4(uint8_t* dst, const int (&q)[E]) {
    if constexpr (E == 8) {
        uint32_t w = pack_nibbles(q[0], q[1]) | (pack_nibbles(q[2], q[3]) << 8) |
                     (pack_nibbles(q[4], q[5]) << 16) | (pack_nibbles(q[6], q[7]) << 24);
        *reinterpret_cast<uint32_t*>(dst) = w;
    } else {
#pragma unroll
        for (int i = 0; i < E / 2; ++i) dst[i] = (uint8_t)pack_nibbles(q[2 * i], q[2 * i + 1]);
    }
}

// ---------------------------------------------------------------------------
// quant_k_int4: per-channel absmax over S, one CTA per (b, h, channel block).
// ---------------------------------------------------------------------------
constexpr int kQuantThreads = 256;

template <int DT, int E>
__global__ void __launch_bounds__(kQuantThreads)
quant_int4_k_kernel(const typename Elem<DT>::T* __restrict__ x, fade_view4 v, int dims_per_cta,
                    uint8_t* __restrict__ packed, typename Elem<DT>::T* __restrict__ scale,
                    bool vec) {
    using T = typename Elem<DT>::T;
    const int z = blockIdx.x;
    const int b = z / (int)v.H, h = z % (int)v.H;
    const int d_lo = blockIdx.y * dims_per_cta;
    const int D = (int)v.D;
    const int tpr = dims_per_cta / E;           // threads per row
    const int rows_per_iter = kQuantThreads / tpr;
    const int slot = threadIdx.x / tpr;
    const int dg = d_lo + (threadIdx.x % tpr) * E;
    const bool active = slot < rows_per_iter && dg < D;
    const T* xb = x + b * v.sb + h * v.sh + (int64_t)dg * v.sd;

    float amax[E];
#pragma unroll
    for (int i = 0; i < E; ++i) amax[i] = 0.f;
    if (active) {
        int64_t s = slot;
        for (; s + 3 * rows_per_iter < v.S; s += 4 * rows_per_iter) {   // four rows in flight
            float e[4][E];
#pragma unroll
            for (int u = 0; u < 4; ++u) load_elems<DT, E>(xb + (s + u * rows_per_iter) * v.ss, v.sd, vec, e[u]);
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
                for (int i = 0; i < E; ++i) amax[i] = fmaxf(amax[i], fabsf(e[u][i]));
        }
        for (; s < v.S; s += rows_per_iter) {
            float e[E];
            load_elems<DT, E>(xb + s * v.ss, v.sd, vec, e);
#pragma unroll
            for (int i = 0; i < E; ++i) amax[i] = fmaxf(amax[i], fabsf(e[i]));
        }
    }
    // Reduce across row slots through shared memory: [rows_per_iter][dims].
    __shared__ float red[kQuantThreads * 8];
#pragma unroll
    for (int i = 0; i < E; ++i) red[threadIdx.x * E + i] = amax[i];
    __syncthreads();
    __shared__ float s_inv[256], s_scale[256];
    for (int c = threadIdx.x; c < dims_per_cta; c += kQuantThreads) {
        const int t = c / E, i = c % E;
        float m = 0.f;
        for (int r = 0; r < rows_per_iter; ++r) m = fmaxf(m, red[(r * tpr + t) * E + i]);
        // absmax.clamp(min=EPS) in the dtype; inv = 7/absmax; scale = absmax/7.
        m = fmaxf(m, Elem<DT>::eps());
        s_inv[c] = inv_scale<DT>(m, 7.f);
        const float sc = Elem<DT>::rnd(__fdiv_rn(m, 7.f));
        s_scale[c] = sc;
        const int d = d_lo + c;
        if (d < D) scale[(int64_t)z * D + d] = Elem<DT>::from_f(sc);
    }
    __syncthreads();
    if (!active) return;
    float inv[E];
#pragma unroll
    for (int i = 0; i < E; ++i) inv[i] = s_inv[dg - d_lo + i];
    uint8_t* pb = packed + (int64_t)z * v.S * (D / 2) + dg / 2;
    int64_t s = slot;
    for (; s + 3 * rows_per_iter < v.S; s += 4 * rows_per_iter) {   // four rows in flight
        float e[4][E];
#pragma unroll
        for (int u = 0; u < 4; ++u) load_elems<DT, E>(xb + (s + u * rows_per_iter) * v.ss, v.sd, vec, e[u]);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            int q[E];
#pragma unroll
            for (int i = 0; i < E; ++i) q[i] = quant_code(Elem<DT>::rnd(__fmul_rn(e[u][i], inv[i])), -8.f, 7.f);
            store_int4<E>(pb + (s + u * rows_per_iter) * (D / 2), q);
        }
    }
    for (; s < v.S; s += rows_per_iter) {
        float e[E];
        load_elems<DT, E>(xb + s * v.ss, v.sd, vec, e);
        int q[E];
#pragma unroll
        for (int i = 0; i < E; ++i) q[i] = quant_code(Elem<DT>::rnd(__fmul_rn(e[i], inv[i])), -8.f, 7.f);
        store_int4<E>(pb + s * (D / 2), q);
    }
}

// ---------------------------------------------------------------------------
// quant_v_int4: per-token absmax over D.  A row is handled by D/E lanes of
// one warp (D <= 256 with E = 8); rows are independent.
// ---------------------------------------------------------------------------
template <int DT, int E>
__global__ void __launch_bounds__(kQuantThreads)
quant_int4_v_kernel(const typename Elem<DT>::T* __restrict__ x, fade_view4 v, int tpr_pow2,
                    uint8_t* __restrict__ packed, typename Elem<DT>::T* __restrict__ scale,
                    bool vec) {
    constexpr int U = 4;       // rows in flight per thread (loads issued before any math)
    const int D = (int)v.D;
    const int tpr = tpr_pow2;  // power of two >= D / E, <= 32
    const int rows_per_cta = kQuantThreads / tpr;
    const int64_t rows = v.B * v.H * v.S;
    const int lane_in_row = threadIdx.x % tpr;
    const bool has_elems = lane_in_row * E < D;
    const int64_t step = (int64_t)gridDim.x * rows_per_cta;
    // rows equally spaced in memory (a contiguous [B, H, S] row space): the
    // row offset is row * ss, no per-row index decomposition
    const bool flat = v.sh == v.S * v.ss && v.sb == v.H * v.sh;
    for (int64_t base = (int64_t)blockIdx.x * rows_per_cta + threadIdx.x / tpr; base < rows; base += U * step) {
        float e[U][E];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t row = base + u * step;
#pragma unroll
            for (int i = 0; i < E; ++i) e[u][i] = 0.f;
            if (row < rows && has_elems) {
                int64_t off;
                if (flat) {
                    off = row * v.ss;
                } else {
                    const int64_t s = row % v.S, bh = row / v.S;
                    const int64_t b = bh / v.H, h = bh % v.H;
                    off = b * v.sb + h * v.sh + s * v.ss;
                }
                load_elems<DT, E>(x + off + (int64_t)lane_in_row * E * v.sd, v.sd, vec, e[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t row = base + u * step;
            float m = 0.f;
#pragma unroll
            for (int i = 0; i < E; ++i) m = fmaxf(m, fabsf(e[u][i]));
            for (int off = tpr / 2; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
            if (row >= rows) continue;
            m = fmaxf(m, Elem<DT>::eps());
            const float inv = inv_scale<DT>(m, 7.f);
            if (lane_in_row == 0) scale[row] = Elem<DT>::from_f(Elem<DT>::rnd(__fdiv_rn(m, 7.f)));
            if (!has_elems) continue;
            int q[E];
#pragma unroll
            for (int i = 0; i < E; ++i) q[i] = quant_code(Elem<DT>::rnd(__fmul_rn(e[u][i], inv)), -8.f, 7.f);
            store_int4<E>(packed + row * (D / 2) + lane_in_row * (E / 2), q);
        }
    }
}

// ---------------------------------------------------------------------------
// Grouped INT2 (fade/quant.py:95-112 / 130-150): one CTA per (b, h, group).
// ---------------------------------------------------------------------------
template <int DT, int E>
__global__ void __launch_bounds__(kQuantThreads)
quant_int2_grouped_kernel(const typename Elem<DT>::T* __restrict__ x, fade_view4 v, int group,
                          int8_t* __restrict__ codes_i8, uint8_t* __restrict__ codes_u8,
                          typename Elem<DT>::T* __restrict__ scale, bool vec) {
    using T = typename Elem<DT>::T;
    const int D = (int)v.D;
    const int64_t G = v.S / group;
    const int64_t zg = blockIdx.x;               // (b*H + h) * G + g
    const int64_t g = zg % G, bh = zg / G;
    const int64_t b = bh / v.H, h = bh % v.H;
    const int tpr = D / E;
    const int rows_per_iter = kQuantThreads / tpr;
    const int slot = threadIdx.x / tpr;
    const int dg = (threadIdx.x % tpr) * E;
    const bool active = slot < rows_per_iter;
    const T* xb = x + b * v.sb + h * v.sh + (g * group) * v.ss + (int64_t)dg * v.sd;

    float amax[E];
#pragma unroll
    for (int i = 0; i < E; ++i) amax[i] = 0.f;
    if (active) {
        for (int s = slot; s < group; s += rows_per_iter) {
            float e[E];
            load_elems<DT, E>(xb + s * v.ss, v.sd, vec, e);
#pragma unroll
            for (int i = 0; i < E; ++i) amax[i] = fmaxf(amax[i], fabsf(e[i]));
        }
    }
    __shared__ float red[kQuantThreads * 8];
#pragma unroll
    for (int i = 0; i < E; ++i) red[threadIdx.x * E + i] = amax[i];
    __syncthreads();
    __shared__ float s_inv[512];
    for (int c = threadIdx.x; c < D; c += kQuantThreads) {
        const int t = c / E, i = c % E;
        float m = 0.f;
        for (int r = 0; r < rows_per_iter; ++r) m = fmaxf(m, red[(r * tpr + t) * E + i]);
        m = fmaxf(m, Elem<DT>::eps());
        s_inv[c] = inv_scale<DT>(m, 1.f);                  // 1 / absmax
        scale[zg * D + c] = Elem<DT>::from_f(Elem<DT>::rnd(__fdiv_rn(m, 1.f)));
    }
    __syncthreads();
    if (!active) return;
    float inv[E];
#pragma unroll
    for (int i = 0; i < E; ++i) inv[i] = s_inv[dg + i];
    const int64_t row0 = bh * v.S + g * group;
    for (int s = slot; s < group; s += rows_per_iter) {
        float e[E];
        load_elems<DT, E>(xb + s * v.ss, v.sd, vec, e);
        int q[E];
#pragma unroll
        for (int i = 0; i < E; ++i) q[i] = quant_code(Elem<DT>::rnd(__fmul_rn(e[i], inv[i])), -2.f, 1.f);
        const int64_t row = row0 + s;
        if (codes_i8) {
#pragma unroll
            for (int i = 0; i < E; ++i) codes_i8[row * D + dg + i] = (int8_t)q[i];
        }
        if (codes_u8) {
            if constexpr (E == 8) {
                uint8_t* dst = codes_u8 + row * (D / 4) + dg / 4;
                dst[0] = (uint8_t)pack_crumbs(q[0], q[1], q[2], q[3]);
                dst[1] = (uint8_t)pack_crumbs(q[4], q[5], q[6], q[7]);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Pack / unpack / dequant (elementwise)
// ---------------------------------------------------------------------------
__global__ void pack_codes_kernel(const int8_t* __restrict__ q, int64_t n_out, int bits,
                                  uint8_t* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_out;
         i += (int64_t)gridDim.x * blockDim.x) {
        if (bits == 4) {
            out[i] = (uint8_t)pack_nibbles(q[2 * i], q[2 * i + 1]);
        } else {
            out[i] = (uint8_t)pack_crumbs(q[4 * i], q[4 * i + 1], q[4 * i + 2], q[4 * i + 3]);
        }
    }
}

__device__ __forceinline__ int sext(uint32_t u, int bits) {
    const uint32_t sign = 1u << (bits - 1);
    return (int)(u & (2 * sign - 1)) - (int)((u & sign) << 1);
}

__global__ void unpack_codes_kernel(const uint8_t* __restrict__ p, int64_t n_in, int bits,
                                    int8_t* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_in;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t byte = p[i];
        if (bits == 4) {
            out[2 * i] = (int8_t)sext(byte >> 4, 4);
            out[2 * i + 1] = (int8_t)sext(byte & 15u, 4);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) out[4 * i + j] = (int8_t)sext((byte >> (6 - 2 * j)) & 3u, 2);
        }
    }
}

__device__ __forceinline__ int code_at(const uint8_t* __restrict__ codes, int bits, int64_t row,
                                       int64_t D, int64_t d) {
    if (bits == 8) return (int)reinterpret_cast<const int8_t*>(codes)[row * D + d];
    if (bits == 4) {
        const uint32_t byte = codes[row * (D / 2) + d / 2];
        return sext((d & 1) ? (byte & 15u) : (byte >> 4), 4);
    }
    const uint32_t byte = codes[row * (D / 4) + d / 4];
    return sext((byte >> (6 - 2 * (d & 3))) & 3u, 2);
}

template <int DT>
__global__ void dequant_kernel(const uint8_t* __restrict__ codes, int bits,
                               const typename Elem<DT>::T* __restrict__ scale, int scale_mode,
                               int group, int64_t H, int64_t S, int64_t D, int64_t n,
                               typename Elem<DT>::T* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t d = i % D, row = i / D;
        const int64_t s = row % S, bh = row / S;
        int64_t si;
        if (scale_mode == 0) si = bh * D + d;
        else if (scale_mode == 1) si = row;
        else si = (bh * (S / group) + s / group) * D + d;
        // q.to(dtype) is exact for these small integers; one rounded multiply.
        const float q = (float)code_at(codes, bits, row, D, d);
        out[i] = Elem<DT>::from_f(__fmul_rn(q, Elem<DT>::to_f(scale[si])));
    }
}

// INT4 with per-channel (mode 0) or per-token (mode 1) scales, D % 8 == 0:
// one thread per 8 codes (one 32-bit code word -> one 16-byte store for
// 16-bit dtypes), grid-stride.  Same rounding as dequant_kernel.
template <int DT>
__global__ void dequant_int4_vec_kernel(const uint32_t* __restrict__ codes,
                                        const typename Elem<DT>::T* __restrict__ scale, int scale_mode,
                                        int64_t S, int D, int64_t n8, typename Elem<DT>::T* __restrict__ out) {
    using T = typename Elem<DT>::T;
    const int w_per_row = D / 8;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / w_per_row;
        const int d0 = (int)(i - row * w_per_row) * 8;
        const uint32_t w = codes[i];
        float sc[8];
        if (scale_mode == 0) {
            const T* sp = scale + (row / S) * D + d0;
#pragma unroll
            for (int j = 0; j < 8; ++j) sc[j] = Elem<DT>::to_f(sp[j]);
        } else {
            const float s1 = Elem<DT>::to_f(scale[row]);
#pragma unroll
            for (int j = 0; j < 8; ++j) sc[j] = s1;
        }
        T o[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t byte = (w >> (8 * j)) & 0xFFu;
            const int hi = (int)((byte >> 4) & 7u) - (int)(byte & 0x80u ? 8 : 0);
            const int lo = (int)(byte & 7u) - (int)(byte & 0x8u ? 8 : 0);
            o[2 * j] = Elem<DT>::from_f(__fmul_rn((float)hi, sc[2 * j]));
            o[2 * j + 1] = Elem<DT>::from_f(__fmul_rn((float)lo, sc[2 * j + 1]));
        }
        T* dst = out + i * 8;
        if constexpr (sizeof(T) == 2) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(o);
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) dst[j] = o[j];
        }
    }
}

// ---------------------------------------------------------------------------
// Age-out: the oldest recent-ring token of every (b, h) joins the INT4 middle;
// the new token takes its ring slot.  One CTA per batch row b, one warp per
// kv head (strided); lane owns channel pairs.
// ---------------------------------------------------------------------------
template <int DT>
__global__ void age_out_int4_kernel(typename Elem<DT>::T* __restrict__ ring_k,
                                    typename Elem<DT>::T* __restrict__ ring_v, int H, int D,
                                    int64_t ring_cap, int64_t ring_sb, int64_t ring_sh,
                                    int64_t ring_origin, uint8_t* __restrict__ k_packed,
                                    uint8_t* __restrict__ v_packed,
                                    typename Elem<DT>::T* __restrict__ v_scale,
                                    const typename Elem<DT>::T* __restrict__ k_scale, int64_t mid_sb,
                                    int64_t mid_sh, int64_t mid_cap, int32_t* __restrict__ mid_len,
                                    const typename Elem<DT>::T* __restrict__ k_new,
                                    const typename Elem<DT>::T* __restrict__ v_new, int64_t new_sb,
                                    int64_t new_sh) {
    griddep_wait();
    const int b = blockIdx.x;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
    const int64_t n = mid_len[b];
    griddep_launch_dependents();
    const bool room = n < mid_cap;
    int64_t slot = (n - ring_origin) % ring_cap;
    if (slot < 0) slot += ring_cap;
    for (int h = warp; h < H; h += nw) {
        auto* ks = ring_k + b * ring_sb + h * ring_sh + slot * D;
        auto* vs = ring_v + b * ring_sb + h * ring_sh + slot * D;
        // the new token does not depend on the slot: fetch it first
        typename Elem<DT>::T kn_r[8], vn_r[8];
        if (k_new) {
            const auto* kn = k_new + b * new_sb + h * new_sh;
            const auto* vn = v_new + b * new_sb + h * new_sh;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int d = lane + 32 * i;
                if (d < D) { kn_r[i] = kn[d]; vn_r[i] = vn[d]; }
            }
        }
        if (room) {
            const auto* sc = k_scale + ((int64_t)b * H + h) * D;
            const int64_t row = b * mid_sb + h * mid_sh + n;
            float m = 0.f;
            for (int d = lane; d < D; d += 32) m = fmaxf(m, fabsf(Elem<DT>::to_f(vs[d])));
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
            m = fmaxf(m, Elem<DT>::eps());
            const float inv = inv_scale<DT>(m, 7.f);
            if (lane == 0) v_scale[row] = Elem<DT>::from_f(Elem<DT>::rnd(__fdiv_rn(m, 7.f)));
            for (int p = lane; p < D / 2; p += 32) {
                int kq[2], vq[2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const int d = 2 * p + j;
                    const float s = Elem<DT>::to_f(sc[d]);
                    const float kx = Elem<DT>::to_f(ks[d]);
                    kq[j] = (s > 0.f) ? quant_code(__fdiv_rn(kx, s), -8.f, 7.f) : 0;
                    vq[j] = quant_code(Elem<DT>::rnd(__fmul_rn(Elem<DT>::to_f(vs[d]), inv)), -8.f, 7.f);
                }
                k_packed[row * (D / 2) + p] = (uint8_t)pack_nibbles(kq[0], kq[1]);
                v_packed[row * (D / 2) + p] = (uint8_t)pack_nibbles(vq[0], vq[1]);
            }
        }
        __syncwarp();
        if (k_new && room) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int d = lane + 32 * i;
                if (d < D) { ks[d] = kn_r[i]; vs[d] = vn_r[i]; }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && room) mid_len[b] = (int32_t)(n + 1);
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
static bool view_ok(const fade_view4& v) {
    return v.B >= 0 && v.H >= 0 && v.S >= 0 && v.D > 0;
}

static bool can_vec(const void* x, const fade_view4& v, int elem_bytes) {
    return v.sd == 1 && aligned16(x) && ((v.sb * elem_bytes) % 16 == 0) &&
           ((v.sh * elem_bytes) % 16 == 0) && ((v.ss * elem_bytes) % 16 == 0);
}

// quant_k_int4 for long rows: a cluster of kKClus CTAs per (b, h) and
// channel part (D / nsplit channels), each CTA over a contiguous slice of S.
// Each CTA reduces the absmax of its slice (kKRows rows in flight per
// thread), the cluster combines the kKClus partial maxima through
// distributed shared memory, and each CTA then quantises its own slice,
// which it read moments before.  With D = 128 split in two halves (128-byte
// row segments) the resident CTAs' slices total less than the 126 MB L2, so
// that second read is an L2 hit rather than a second trip to HBM.
constexpr int kKClus = 8;
constexpr int kKRows = 4;

template <int DT>
__global__ void __cluster_dims__(kKClus, 1, 1) __launch_bounds__(kQuantThreads)
quant_int4_k_cluster_kernel(const typename Elem<DT>::T* __restrict__ x, fade_view4 v, uint8_t* __restrict__ packed,
                            typename Elem<DT>::T* __restrict__ scale, bool vec, int nsplit) {
    using T = typename Elem<DT>::T;
    constexpr int E = 8, U = kKRows;
    const int cid = blockIdx.x / kKClus, rank = blockIdx.x % kKClus;
    const int z = cid / nsplit;
    const int b = z / (int)v.H, h = z % (int)v.H;
    const int Dfull = (int)v.D;
    const int D = Dfull / nsplit;                // this cluster's channels: [c0, c0 + D)
    const int c0 = (cid % nsplit) * D;
    const int tpr = D / E;                       // threads per row (D <= 256: tpr <= 32)
    const int rows_per_iter = kQuantThreads / tpr;
    const int slot = threadIdx.x / tpr;
    const int dg = (threadIdx.x % tpr) * E;
    const int64_t s0 = v.S * rank / kKClus, s1 = v.S * (rank + 1) / kKClus;
    const T* xb = x + b * v.sb + h * v.sh + (int64_t)(c0 + dg) * v.sd;

    float amax[E];
#pragma unroll
    for (int i = 0; i < E; ++i) amax[i] = 0.f;
    int64_t s = s0 + slot;
    for (; s + (U - 1) * rows_per_iter < s1; s += U * rows_per_iter) {
        float e[U][E];
#pragma unroll
        for (int u = 0; u < U; ++u) load_elems<DT, E>(xb + (s + u * rows_per_iter) * v.ss, v.sd, vec, e[u]);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int i = 0; i < E; ++i) amax[i] = fmaxf(amax[i], fabsf(e[u][i]));
    }
    for (; s < s1; s += rows_per_iter) {
        float e[E];
        load_elems<DT, E>(xb + s * v.ss, v.sd, vec, e);
#pragma unroll
        for (int i = 0; i < E; ++i) amax[i] = fmaxf(amax[i], fabsf(e[i]));
    }
    __shared__ float red[kQuantThreads * E];
    __shared__ float camax[256];                 // this CTA's per-channel maxima
    __shared__ float s_inv[256];
#pragma unroll
    for (int i = 0; i < E; ++i) red[threadIdx.x * E + i] = amax[i];
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += kQuantThreads) {
        const int t = c / E, i = c % E;
        float m = 0.f;
        for (int r = 0; r < rows_per_iter; ++r) m = fmaxf(m, red[(r * tpr + t) * E + i]);
        camax[c] = m;
    }
    // cluster-wide maxima: read every member's camax (distributed shared memory)
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    const uint32_t local = (uint32_t)__cvta_generic_to_shared(camax);
    for (int c = threadIdx.x; c < D; c += kQuantThreads) {
        float m = 0.f;
#pragma unroll
        for (int r = 0; r < kKClus; ++r) {
            uint32_t remote;
            float val;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local + 4u * c), "r"(r));
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(val) : "r"(remote) : "memory");
            m = fmaxf(m, val);
        }
        // absmax.clamp(min=EPS) in the dtype; inv = 7/absmax; scale = absmax/7.
        m = fmaxf(m, Elem<DT>::eps());
        s_inv[c] = inv_scale<DT>(m, 7.f);
        if (rank == 0) scale[(int64_t)z * Dfull + c0 + c] = Elem<DT>::from_f(Elem<DT>::rnd(__fdiv_rn(m, 7.f)));
    }
    // no member leaves (or reuses camax) while another may still read it
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    float inv[E];
#pragma unroll
    for (int i = 0; i < E; ++i) inv[i] = s_inv[dg + i];
    uint8_t* pb = packed + (int64_t)z * v.S * (Dfull / 2) + (c0 + dg) / 2;
    s = s0 + slot;
    for (; s + (U - 1) * rows_per_iter < s1; s += U * rows_per_iter) {
        float e[U][E];
#pragma unroll
        for (int u = 0; u < U; ++u) load_elems<DT, E>(xb + (s + u * rows_per_iter) * v.ss, v.sd, vec, e[u]);
#pragma unroll
        for (int u = 0; u < U; ++u) {
            int q[E];
#pragma unroll
            for (int i = 0; i < E; ++i) q[i] = quant_code(Elem<DT>::rnd(__fmul_rn(e[u][i], inv[i])), -8.f, 7.f);
            store_int4<E>(pb + (s + u * rows_per_iter) * (Dfull / 2), q);
        }
    }
    for (; s < s1; s += rows_per_iter) {
        float e[E];
        load_elems<DT, E>(xb + s * v.ss, v.sd, vec, e);
        int q[E];
#pragma unroll
        for (int i = 0; i < E; ++i) q[i] = quant_code(Elem<DT>::rnd(__fmul_rn(e[i], inv[i])), -8.f, 7.f);
        store_int4<E>(pb + s * (Dfull / 2), q);
    }
}

template <int DT>
static int launch_quant_k(const void* x, const fade_view4& v, uint8_t* packed, void* scale,
                          cudaStream_t st) {
    using T = typename Elem<DT>::T;
    const int64_t Z = v.B * v.H;
    if (Z == 0 || v.S == 0) {
        // Empty sequence axis: absmax is the clamped EPS for every channel.
        if (Z == 0) return FADE_OK;
    }
    const bool e8 = (v.D % 8 == 0);
    if (e8 && v.D <= 256 && v.S >= 64 * kKClus) {
        const bool vec = can_vec(x, v, sizeof(T));
        // two channel halves when each stays a whole 128-byte row segment
        const int nsplit = (v.D % 16 == 0 && v.D / 2 * (int64_t)sizeof(T) >= 128) ? 2 : 1;
        quant_int4_k_cluster_kernel<DT><<<(unsigned)(Z * nsplit * kKClus), kQuantThreads, 0, st>>>(
            (const T*)x, v, packed, (T*)scale, vec, nsplit);
        FADE_LAUNCH_CHECK();
        return FADE_OK;
    }
    const int E = e8 ? 8 : 2;
    int dims_per_cta = (int)(v.D < 256 ? v.D : 256);
    // For few (b,h) pairs, split channels across CTAs to fill the machine.
    // (blocks of at least 64 channels: 128-byte row segments; narrower ones
    // double the DRAM sectors fetched per useful byte)
    while (Z * (v.D / dims_per_cta) < 148 && dims_per_cta > 8 * E && dims_per_cta % (2 * E) == 0 &&
           (dims_per_cta / 2) % E == 0 && v.D % (dims_per_cta / 2) == 0)
        dims_per_cta /= 2;
    dim3 grid((unsigned)Z, (unsigned)((v.D + dims_per_cta - 1) / dims_per_cta));
    const bool vec = e8 && can_vec(x, v, sizeof(T));
    if (e8)
        quant_int4_k_kernel<DT, 8><<<grid, kQuantThreads, 0, st>>>(
            (const T*)x, v, dims_per_cta, packed, (T*)scale, vec);
    else
        quant_int4_k_kernel<DT, 2><<<grid, kQuantThreads, 0, st>>>(
            (const T*)x, v, dims_per_cta, packed, (T*)scale, false);
    FADE_LAUNCH_CHECK();
    return FADE_OK;
}

template <int DT>
static int launch_quant_v(const void* x, const fade_view4& v, uint8_t* packed, void* scale,
                          cudaStream_t st) {
    using T = typename Elem<DT>::T;
    const int64_t rows = v.B * v.H * v.S;
    if (rows == 0) return FADE_OK;
    const int E = (v.D % 8 == 0) ? 8 : 2;
    int tpr = 1;
    while (tpr * E < v.D) tpr *= 2;
    if (tpr > 32) return FADE_ERR_UNSUPPORTED;
    const int rows_per_cta = kQuantThreads / tpr;
    int64_t g = (rows + rows_per_cta - 1) / rows_per_cta;
    if (g > 148 * 8) g = 148 * 8;   // resident grid; each thread keeps 4 rows in flight
    const unsigned grid = (unsigned)g;
    if (E == 8)
        quant_int4_v_kernel<DT, 8><<<grid, kQuantThreads, 0, st>>>(
            (const T*)x, v, tpr, packed, (T*)scale, can_vec(x, v, sizeof(T)));
    else
        quant_int4_v_kernel<DT, 2><<<grid, kQuantThreads, 0, st>>>(
            (const T*)x, v, tpr, packed, (T*)scale, false);
    FADE_LAUNCH_CHECK();
    return FADE_OK;
}

// Grouped INT2 at head_dim 128 for groups of up to 32 rows: one warp per
// (b, h, group).  Lanes 0-15 hold the even rows, 16-31 the odd rows, 8
// channels each; the group's rows stay in registers (raw 16-byte loads, all
// issued before any math), the per-channel absmax is one shuffle across the
// two halves, and the codes are made from the registers: one HBM read, no
// shared memory and no block barrier.
constexpr int kInt2MaxRows = 32;

template <int DT>
__global__ void __launch_bounds__(256, 2)
quant_int2_grouped_warp_kernel(const typename Elem<DT>::T* __restrict__ x, fade_view4 v, int group,
                               int64_t n_groups, int8_t* __restrict__ codes_i8, uint8_t* __restrict__ codes_u8,
                               typename Elem<DT>::T* __restrict__ scale) {
    using T = typename Elem<DT>::T;
    constexpr int E = 8, D = 128, RMAX = kInt2MaxRows / 2;
    const int64_t zg = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;   // (b*H + h) * G + g
    if (zg >= n_groups) return;
    const int lane = threadIdx.x % 32, half = lane >> 4, t = lane & 15;
    const int64_t G = v.S / group;
    const int64_t g = zg % G, bh = zg / G;
    const int64_t b = bh / v.H, h = bh % v.H;
    const T* xb = x + b * v.sb + h * v.sh + (g * group + half) * v.ss + (int64_t)t * E;
    const int R = group / 2;
    uint4 raw[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; ++r)
        if (r < R) raw[r] = __ldg(reinterpret_cast<const uint4*>(xb + (int64_t)(2 * r) * v.ss));
    float amax[E];
#pragma unroll
    for (int i = 0; i < E; ++i) amax[i] = 0.f;
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
        if (r < R) {
            const T* e = reinterpret_cast<const T*>(&raw[r]);
#pragma unroll
            for (int i = 0; i < E; ++i) amax[i] = fmaxf(amax[i], fabsf(Elem<DT>::to_f(e[i])));
        }
    }
    float inv[E];
    uint4 sw;
    T* so = reinterpret_cast<T*>(&sw);
#pragma unroll
    for (int i = 0; i < E; ++i) {
        float m = fmaxf(amax[i], __shfl_xor_sync(0xffffffffu, amax[i], 16));
        m = fmaxf(m, Elem<DT>::eps());
        inv[i] = inv_scale<DT>(m, 1.f);                   // 1 / absmax
        so[i] = Elem<DT>::from_f(Elem<DT>::rnd(__fdiv_rn(m, 1.f)));
    }
    if (half == 0) *reinterpret_cast<uint4*>(scale + zg * D + t * E) = sw;
    const int64_t row0 = bh * v.S + g * group + half;
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
        if (r < R) {
            const T* e = reinterpret_cast<const T*>(&raw[r]);
            int q[E];
#pragma unroll
            for (int i = 0; i < E; ++i) q[i] = quant_code(Elem<DT>::rnd(__fmul_rn(Elem<DT>::to_f(e[i]), inv[i])), -2.f, 1.f);
            const int64_t row = row0 + 2 * r;
            if (codes_i8) {
                uint2 w;
                w.x = (uint32_t)(q[0] & 0xFF) | ((uint32_t)(q[1] & 0xFF) << 8) | ((uint32_t)(q[2] & 0xFF) << 16) |
                      ((uint32_t)(q[3] & 0xFF) << 24);
                w.y = (uint32_t)(q[4] & 0xFF) | ((uint32_t)(q[5] & 0xFF) << 8) | ((uint32_t)(q[6] & 0xFF) << 16) |
                      ((uint32_t)(q[7] & 0xFF) << 24);
                *reinterpret_cast<uint2*>(codes_i8 + row * D + t * E) = w;
            }
            if (codes_u8) {
                const uint32_t w = pack_crumbs(q[0], q[1], q[2], q[3]) | (pack_crumbs(q[4], q[5], q[6], q[7]) << 8);
                *reinterpret_cast<uint16_t*>(codes_u8 + row * (D / 4) + t * 2) = (uint16_t)w;
            }
        }
    }
}

template <int DT>
static int launch_int2(const void* x, const fade_view4& v, int group, int8_t* ci8, uint8_t* cu8,
                       void* scale, cudaStream_t st) {
    using T = typename Elem<DT>::T;
    const int64_t n = v.B * v.H * (v.S / group);
    if (n == 0) return FADE_OK;
    if constexpr (DT != FADE_F32) {
        // warp per group: D = 128, even group <= 32, 16-byte rows, 8-byte code rows
        if (v.D == 128 && group % 2 == 0 && group <= kInt2MaxRows && can_vec(x, v, sizeof(T)) &&
            (v.ss * (int64_t)sizeof(T)) % 16 == 0 && ((uintptr_t)ci8 % 8) == 0 && ((uintptr_t)cu8 % 2) == 0 &&
            ((uintptr_t)scale % 16) == 0) {
            quant_int2_grouped_warp_kernel<DT><<<(unsigned)((n + 7) / 8), 256, 0, st>>>(
                (const T*)x, v, group, n, ci8, cu8, (T*)scale);
            FADE_LAUNCH_CHECK();
            return FADE_OK;
        }
    }
    if (v.D % 8 != 0 || v.D / 8 > kQuantThreads || v.D > 512) {
        if (cu8) return FADE_ERR_UNSUPPORTED;
        if (v.D / 2 > kQuantThreads) return FADE_ERR_UNSUPPORTED;
        quant_int2_grouped_kernel<DT, 2><<<(unsigned)n, kQuantThreads, 0, st>>>(
            (const T*)x, v, group, ci8, cu8, (T*)scale, false);
    } else {
        quant_int2_grouped_kernel<DT, 8><<<(unsigned)n, kQuantThreads, 0, st>>>(
            (const T*)x, v, group, ci8, cu8, (T*)scale, can_vec(x, v, sizeof(T)));
    }
    FADE_LAUNCH_CHECK();
    return FADE_OK;
}

static unsigned ew_grid(int64_t n) {
    int64_t g = (n + 255) / 256;
    if (g > 148 * 32) g = 148 * 32;
    if (g < 1) g = 1;
    return (unsigned)g;
}

}  // namespace fade

using namespace fade;

extern "C" int fade_quant_int4_k(const void* x, int dtype, fade_view4 xv, uint8_t* packed,
                                 void* scale, void* stream) {
    if (!view_ok(xv)) return FADE_ERR_INVALID_ARG;
    if (xv.D % 2 != 0) return FADE_ERR_ODD_DIM;
    if (xv.B * xv.H == 0) return FADE_OK;
    if (!x || !packed || !scale) return FADE_ERR_INVALID_ARG;
    if (xv.D > 4096) return FADE_ERR_UNSUPPORTED;
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case FADE_F16: return launch_quant_k<FADE_F16>(x, xv, packed, scale, st);
        case FADE_BF16: return launch_quant_k<FADE_BF16>(x, xv, packed, scale, st);
        case FADE_F32: return launch_quant_k<FADE_F32>(x, xv, packed, scale, st);
    }
    return FADE_ERR_INVALID_ARG;
}

extern "C" int fade_quant_int4_v(const void* x, int dtype, fade_view4 xv, uint8_t* packed,
                                 void* scale, void* stream) {
    if (!view_ok(xv)) return FADE_ERR_INVALID_ARG;
    if (xv.D % 2 != 0) return FADE_ERR_ODD_DIM;
    if (xv.B * xv.H * xv.S == 0) return FADE_OK;
    if (!x || !packed || !scale) return FADE_ERR_INVALID_ARG;
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case FADE_F16: return launch_quant_v<FADE_F16>(x, xv, packed, scale, st);
        case FADE_BF16: return launch_quant_v<FADE_BF16>(x, xv, packed, scale, st);
        case FADE_F32: return launch_quant_v<FADE_F32>(x, xv, packed, scale, st);
    }
    return FADE_ERR_INVALID_ARG;
}

extern "C" int fade_quant_int2_grouped(const void* x, int dtype, fade_view4 xv, int group,
                                       int8_t* codes_i8, uint8_t* codes_u8, void* scale,
                                       void* stream) {
    if (!view_ok(xv) || group < 1) return FADE_ERR_INVALID_ARG;
    if (xv.S % group != 0) return FADE_ERR_GROUP;
    if (codes_u8 && xv.D % 4 != 0) return FADE_ERR_ODD_DIM;
    if (xv.B * xv.H * xv.S == 0) return FADE_OK;
    if (!x || !scale || (!codes_i8 && !codes_u8)) return FADE_ERR_INVALID_ARG;
    cudaStream_t st = as_stream(stream);
    switch (dtype) {
        case FADE_F16: return launch_int2<FADE_F16>(x, xv, group, codes_i8, codes_u8, scale, st);
        case FADE_BF16: return launch_int2<FADE_BF16>(x, xv, group, codes_i8, codes_u8, scale, st);
        case FADE_F32: return launch_int2<FADE_F32>(x, xv, group, codes_i8, codes_u8, scale, st);
    }
    return FADE_ERR_INVALID_ARG;
}

extern "C" int fade_pack_codes(const int8_t* q, int64_t rows, int64_t D, int bits, uint8_t* out,
                               void* stream) {
    if (rows < 0 || D < 0 || (bits != 4 && bits != 2)) return FADE_ERR_INVALID_ARG;
    if (D % (8 / bits) != 0) return FADE_ERR_ODD_DIM;
    const int64_t n_out = rows * D * bits / 8;
    if (n_out == 0) return FADE_OK;
    if (!q || !out) return FADE_ERR_INVALID_ARG;
    pack_codes_kernel<<<ew_grid(n_out), 256, 0, as_stream(stream)>>>(q, n_out, bits, out);
    FADE_LAUNCH_CHECK();
    return FADE_OK;
}

extern "C" int fade_unpack_codes(const uint8_t* packed, int64_t rows, int64_t D, int bits,
                                 int8_t* out, void* stream) {
    if (rows < 0 || D < 0 || (bits != 4 && bits != 2)) return FADE_ERR_INVALID_ARG;
    if (D % (8 / bits) != 0) return FADE_ERR_ODD_DIM;
    const int64_t n_in = rows * D * bits / 8;
    if (n_in == 0) return FADE_OK;
    if (!packed || !out) return FADE_ERR_INVALID_ARG;
    unpack_codes_kernel<<<ew_grid(n_in), 256, 0, as_stream(stream)>>>(packed, n_in, bits, out);
    FADE_LAUNCH_CHECK();
    return FADE_OK;
}

extern "C" int fade_dequant(const void* codes, int bits, const void* scale, int scale_mode,
                            int group, int dtype, int64_t B, int64_t H, int64_t S, int64_t D,
                            void* out, void* stream) {
    if (B < 0 || H < 0 || S < 0 || D <= 0) return FADE_ERR_INVALID_ARG;
    if (bits != 8 && bits != 4 && bits != 2) return FADE_ERR_INVALID_ARG;
    if (scale_mode < 0 || scale_mode > 2) return FADE_ERR_INVALID_ARG;
    if (scale_mode == 2 && (group < 1)) return FADE_ERR_INVALID_ARG;
    if (scale_mode == 2 && S % group != 0) return FADE_ERR_GROUP;
    if (D % (8 / (bits == 8 ? 8 : bits)) != 0) return FADE_ERR_ODD_DIM;
    const int64_t n = B * H * S * D;
    if (n == 0) return FADE_OK;
    if (!codes || !scale || !out) return FADE_ERR_INVALID_ARG;
    const auto* c = reinterpret_cast<const uint8_t*>(codes);
    cudaStream_t st = as_stream(stream);
    if (bits == 4 && scale_mode != 2 && D % 8 == 0 && dtype != FADE_F32 &&
        reinterpret_cast<uintptr_t>(codes) % 4 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0) {
        const int64_t n8 = n / 8;
        int64_t g = (n8 + 255) / 256;
        if (g > 148 * 16) g = 148 * 16;
        if (dtype == FADE_F16)
            dequant_int4_vec_kernel<FADE_F16><<<(unsigned)g, 256, 0, st>>>(
                reinterpret_cast<const uint32_t*>(codes), (const __half*)scale, scale_mode, S, (int)D, n8,
                (__half*)out);
        else
            dequant_int4_vec_kernel<FADE_BF16><<<(unsigned)g, 256, 0, st>>>(
                reinterpret_cast<const uint32_t*>(codes), (const __nv_bfloat16*)scale, scale_mode, S, (int)D, n8,
                (__nv_bfloat16*)out);
        FADE_LAUNCH_CHECK();
        return FADE_OK;
    }
    switch (dtype) {
        case FADE_F16:
            dequant_kernel<FADE_F16><<<ew_grid(n), 256, 0, st>>>(
                c, bits, (const __half*)scale, scale_mode, group, H, S, D, n, (__half*)out);
            break;
        case FADE_BF16:
            dequant_kernel<FADE_BF16><<<ew_grid(n), 256, 0, st>>>(
                c, bits, (const __nv_bfloat16*)scale, scale_mode, group, H, S, D, n,
                (__nv_bfloat16*)out);
            break;
        case FADE_F32:
            dequant_kernel<FADE_F32><<<ew_grid(n), 256, 0, st>>>(
                c, bits, (const float*)scale, scale_mode, group, H, S, D, n, (float*)out);
            break;
        default: return FADE_ERR_INVALID_ARG;
    }
    FADE_LAUNCH_CHECK();
    return FADE_OK;
}

extern "C" int fade_age_out_int4(void* ring_k, void* ring_v, int dtype, int64_t B, int64_t H,
                                 int64_t D, int64_t ring_cap, int64_t ring_sb, int64_t ring_sh,
                                 int64_t ring_origin, uint8_t* k_packed, uint8_t* v_packed,
                                 void* v_scale, const void* k_scale, int64_t mid_sb, int64_t mid_sh,
                                 int64_t mid_cap, int32_t* mid_len, const void* k_new,
                                 const void* v_new, int64_t new_sb, int64_t new_sh, void* stream) {
    if (B < 0 || H < 0 || D <= 0 || ring_cap <= 0 || mid_cap < 0) return FADE_ERR_INVALID_ARG;
    if (D % 2 != 0) return FADE_ERR_ODD_DIM;
    if (B * H == 0) return FADE_OK;
    if (!ring_k || !ring_v || !k_packed || !v_packed || !v_scale || !k_scale || !mid_len)
        return FADE_ERR_INVALID_ARG;
    if ((k_new == nullptr) != (v_new == nullptr)) return FADE_ERR_INVALID_ARG;
    if (D > 256) return FADE_ERR_UNSUPPORTED;
    const int threads = (int)(H < 8 ? (H < 1 ? 1 : H) : 8) * 32;
    cudaStream_t st = as_stream(stream);
    void* fn;
    if (dtype == FADE_F16) fn = (void*)&age_out_int4_kernel<FADE_F16>;
    else if (dtype == FADE_BF16) fn = (void*)&age_out_int4_kernel<FADE_BF16>;
    else return FADE_ERR_INVALID_ARG;
    int Hi = (int)H, Di = (int)D;
    void* args[] = {&ring_k, &ring_v, &Hi, &Di, &ring_cap, &ring_sb, &ring_sh, &ring_origin,
                    &k_packed, &v_packed, &v_scale, (void*)&k_scale, &mid_sb, &mid_sh, &mid_cap,
                    &mid_len, (void*)&k_new, (void*)&v_new, &new_sb, &new_sh};
    // programmatic dependent launch: the kernel waits (griddepcontrol.wait)
    // for the previous grid before touching memory, so only its launch overlaps
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)B);
    cfg.blockDim = dim3((unsigned)threads);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    FADE_CUDA_TRY(cudaLaunchKernelExC(&cfg, fn, args));
    return FADE_OK;
}
