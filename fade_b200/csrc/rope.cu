// K3: gather + un-RoPE + re-RoPE for eviction survivors, one pass.
//
// The reference (fade/cache.py:914-935) un-RoPEs all S tokens at their old
// positions (_inverse_rope, fade/cache.py:301-311), index_selects the kept
// ones, then re-RoPEs them at 0..n_kept-1 (_apply_rope, fade/cache.py:290-299).
// Each of its steps is a separate fp32 elementwise op, so
//   pre  = rnd_dt( fp32(k)*cos_old  -  rot(fp32(k))*sin_old )
//   out  = rnd_dt( fp32(pre)*cos_new +  rot(fp32(pre))*sin_new )
// with rot(x)[d] = -x[d+D/2] (d < D/2), x[d-D/2] (d >= D/2), every product and
// sum rounded separately (no FMA contraction).  Only the kept rows are touched.
#include "common.cuh"

namespace fade {

template <int DT>
__global__ void rerope_gather_kernel(const typename Elem<DT>::T* __restrict__ k_in,
                                     const typename Elem<DT>::T* __restrict__ v_in, fade_view4 kv,
                                     const int64_t* __restrict__ keep, int64_t n_kept,
                                     const float* __restrict__ cos_old, const float* __restrict__ sin_old,
                                     const float* __restrict__ cos_new, const float* __restrict__ sin_new,
                                     int apply_rope, typename Elem<DT>::T* __restrict__ k_out,
                                     typename Elem<DT>::T* __restrict__ v_out) {
    const int64_t D = kv.D, half = D / 2;
    const int64_t n = kv.B * kv.H * n_kept * half;
    for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < n;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int64_t d = idx % half;
        const int64_t row = idx / half;  // (b*H + h)*n_kept + i
        const int64_t i = row % n_kept, bh = row / n_kept;
        const int64_t b = bh / kv.H, h = bh % kv.H;
        const int64_t s = keep[i];
        const int64_t src = b * kv.sb + h * kv.sh + s * kv.ss;
        const int64_t dst = row * D;
        const float x1 = Elem<DT>::to_f(k_in[src + d * kv.sd]);
        const float x2 = Elem<DT>::to_f(k_in[src + (d + half) * kv.sd]);
        float y1 = x1, y2 = x2;
        if (apply_rope) {
            const float c1 = cos_old[s * D + d], c2 = cos_old[s * D + d + half];
            const float s1 = sin_old[s * D + d], s2 = sin_old[s * D + d + half];
            // inverse: x*cos - rot(x)*sin ; rot(x) = (-x2, x1)
            const float p1 = Elem<DT>::rnd(__fsub_rn(__fmul_rn(x1, c1), __fmul_rn(-x2, s1)));
            const float p2 = Elem<DT>::rnd(__fsub_rn(__fmul_rn(x2, c2), __fmul_rn(x1, s2)));
            const float n1 = cos_new[i * D + d], n2 = cos_new[i * D + d + half];
            const float m1 = sin_new[i * D + d], m2 = sin_new[i * D + d + half];
            // apply: x*cos + rot(x)*sin
            y1 = __fadd_rn(__fmul_rn(p1, n1), __fmul_rn(-p2, m1));
            y2 = __fadd_rn(__fmul_rn(p2, n2), __fmul_rn(p1, m2));
        }
        k_out[dst + d] = Elem<DT>::from_f(y1);
        k_out[dst + d + half] = Elem<DT>::from_f(y2);
        if (v_in && v_out) {
            v_out[dst + d] = v_in[src + d * kv.sd];
            v_out[dst + d + half] = v_in[src + (d + half) * kv.sd];
        }
    }
}

// Vectorised form for 16-bit K/V rows contiguous in D (the usual layout):
// one thread per 4 channel pairs (d..d+3, d+D/2..d+D/2+3) of one kept row,
// 8-byte K/V and 16-byte cos/sin loads, the row index computed once per
// thread.  Per element the arithmetic is the generic kernel's.
template <int DT>
__global__ void rerope_gather_vec_kernel(const typename Elem<DT>::T* __restrict__ k_in,
                                         const typename Elem<DT>::T* __restrict__ v_in, fade_view4 kv,
                                         const int64_t* __restrict__ keep, int64_t n_kept,
                                         const float* __restrict__ cos_old, const float* __restrict__ sin_old,
                                         const float* __restrict__ cos_new, const float* __restrict__ sin_new,
                                         int apply_rope, int tpr_log2, typename Elem<DT>::T* __restrict__ k_out,
                                         typename Elem<DT>::T* __restrict__ v_out) {
    using T = typename Elem<DT>::T;
    const int D = (int)kv.D, half = D / 2;
    const int64_t rows = kv.B * kv.H * n_kept;
    const int per_block = blockDim.x >> tpr_log2;
    const int64_t row = (int64_t)blockIdx.x * per_block + (threadIdx.x >> tpr_log2);
    if (row >= rows) return;
    const int d = (threadIdx.x & ((1 << tpr_log2) - 1)) * 4;
    const int64_t i = row % n_kept, bh = row / n_kept;
    const int64_t b = bh / kv.H, h = bh % kv.H;
    const int64_t s = keep[i];
    const int64_t src = b * kv.sb + h * kv.sh + s * kv.ss;
    const int64_t dst = row * D;
    const uint2 a = *reinterpret_cast<const uint2*>(k_in + src + d);
    const uint2 c = *reinterpret_cast<const uint2*>(k_in + src + d + half);
    const T* x1v = reinterpret_cast<const T*>(&a);
    const T* x2v = reinterpret_cast<const T*>(&c);
    uint2 oa = a, oc = c;
    T* y1v = reinterpret_cast<T*>(&oa);
    T* y2v = reinterpret_cast<T*>(&oc);
    if (apply_rope) {
        const float4 c1 = *reinterpret_cast<const float4*>(cos_old + s * D + d);
        const float4 c2 = *reinterpret_cast<const float4*>(cos_old + s * D + d + half);
        const float4 s1 = *reinterpret_cast<const float4*>(sin_old + s * D + d);
        const float4 s2 = *reinterpret_cast<const float4*>(sin_old + s * D + d + half);
        const float4 n1 = *reinterpret_cast<const float4*>(cos_new + i * D + d);
        const float4 n2 = *reinterpret_cast<const float4*>(cos_new + i * D + d + half);
        const float4 m1 = *reinterpret_cast<const float4*>(sin_new + i * D + d);
        const float4 m2 = *reinterpret_cast<const float4*>(sin_new + i * D + d + half);
        const float c1a[4] = {c1.x, c1.y, c1.z, c1.w}, c2a[4] = {c2.x, c2.y, c2.z, c2.w};
        const float s1a[4] = {s1.x, s1.y, s1.z, s1.w}, s2a[4] = {s2.x, s2.y, s2.z, s2.w};
        const float n1a[4] = {n1.x, n1.y, n1.z, n1.w}, n2a[4] = {n2.x, n2.y, n2.z, n2.w};
        const float m1a[4] = {m1.x, m1.y, m1.z, m1.w}, m2a[4] = {m2.x, m2.y, m2.z, m2.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float x1 = Elem<DT>::to_f(x1v[j]), x2 = Elem<DT>::to_f(x2v[j]);
            const float p1 = Elem<DT>::rnd(__fsub_rn(__fmul_rn(x1, c1a[j]), __fmul_rn(-x2, s1a[j])));
            const float p2 = Elem<DT>::rnd(__fsub_rn(__fmul_rn(x2, c2a[j]), __fmul_rn(x1, s2a[j])));
            y1v[j] = Elem<DT>::from_f(__fadd_rn(__fmul_rn(p1, n1a[j]), __fmul_rn(-p2, m1a[j])));
            y2v[j] = Elem<DT>::from_f(__fadd_rn(__fmul_rn(p2, n2a[j]), __fmul_rn(p1, m2a[j])));
        }
    }
    *reinterpret_cast<uint2*>(k_out + dst + d) = oa;
    *reinterpret_cast<uint2*>(k_out + dst + d + half) = oc;
    if (v_in && v_out) {
        *reinterpret_cast<uint2*>(v_out + dst + d) = *reinterpret_cast<const uint2*>(v_in + src + d);
        *reinterpret_cast<uint2*>(v_out + dst + d + half) = *reinterpret_cast<const uint2*>(v_in + src + d + half);
    }
}

}  // namespace fade

using namespace fade;

extern "C" int fade_rerope_gather(const void* k_in, const void* v_in, int dtype, fade_view4 kv,
                                  const int64_t* keep_idx, int64_t n_kept, const float* cos_old,
                                  const float* sin_old, const float* cos_new, const float* sin_new,
                                  int apply_rope, void* k_out, void* v_out, void* stream) {
    if (kv.B < 0 || kv.H < 0 || kv.S < 0 || kv.D <= 0 || n_kept < 0) return FADE_ERR_INVALID_ARG;
    if (kv.D % 2 != 0) return FADE_ERR_ODD_DIM;
    const int64_t n = kv.B * kv.H * n_kept * (kv.D / 2);
    if (n == 0) return FADE_OK;
    if (!k_in || !keep_idx || !k_out) return FADE_ERR_INVALID_ARG;
    if (apply_rope && (!cos_old || !sin_old || !cos_new || !sin_new)) return FADE_ERR_INVALID_ARG;
    if ((v_in == nullptr) != (v_out == nullptr)) return FADE_ERR_INVALID_ARG;
    cudaStream_t st = as_stream(stream);
    // vectorised path: 16-bit rows contiguous in D, 8-byte aligned rows and
    // 16-byte aligned tables, D/2 a multiple of 4 with a power-of-two number of
    // 4-pair chunks per row
    const int64_t half = kv.D / 2;
    const int64_t chunks = half / 4;
    const bool pow2 = chunks > 0 && chunks <= 256 && (chunks & (chunks - 1)) == 0;
    auto al = [](const void* p, int a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; };
    if (dtype != FADE_F32 && kv.sd == 1 && half % 4 == 0 && pow2 && kv.sb % 4 == 0 && kv.sh % 4 == 0 &&
        kv.ss % 4 == 0 && al(k_in, 8) && al(k_out, 8) && (!v_in || (al(v_in, 8) && al(v_out, 8))) &&
        (!apply_rope || (al(cos_old, 16) && al(sin_old, 16) && al(cos_new, 16) && al(sin_new, 16)))) {
        int tl = 0;
        while ((1LL << tl) < chunks) ++tl;
        const int per_block = 256 / (int)chunks;
        const int64_t rows = kv.B * kv.H * n_kept;
        const unsigned grid = (unsigned)((rows + per_block - 1) / per_block);
        if (dtype == FADE_F16)
            rerope_gather_vec_kernel<FADE_F16><<<grid, 256, 0, st>>>(
                (const __half*)k_in, (const __half*)v_in, kv, keep_idx, n_kept, cos_old, sin_old, cos_new,
                sin_new, apply_rope, tl, (__half*)k_out, (__half*)v_out);
        else if (dtype == FADE_BF16)
            rerope_gather_vec_kernel<FADE_BF16><<<grid, 256, 0, st>>>(
                (const __nv_bfloat16*)k_in, (const __nv_bfloat16*)v_in, kv, keep_idx, n_kept, cos_old, sin_old,
                cos_new, sin_new, apply_rope, tl, (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out);
        else
            return FADE_ERR_INVALID_ARG;
        FADE_LAUNCH_CHECK();
        return FADE_OK;
    }
    int64_t g = (n + 255) / 256;
    if (g > 148 * 16) g = 148 * 16;
    switch (dtype) {
        case FADE_F16:
            rerope_gather_kernel<FADE_F16><<<(unsigned)g, 256, 0, st>>>(
                (const __half*)k_in, (const __half*)v_in, kv, keep_idx, n_kept, cos_old, sin_old,
                cos_new, sin_new, apply_rope, (__half*)k_out, (__half*)v_out);
            break;
        case FADE_BF16:
            rerope_gather_kernel<FADE_BF16><<<(unsigned)g, 256, 0, st>>>(
                (const __nv_bfloat16*)k_in, (const __nv_bfloat16*)v_in, kv, keep_idx, n_kept, cos_old,
                sin_old, cos_new, sin_new, apply_rope, (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out);
            break;
        case FADE_F32:
            rerope_gather_kernel<FADE_F32><<<(unsigned)g, 256, 0, st>>>(
                (const float*)k_in, (const float*)v_in, kv, keep_idx, n_kept, cos_old, sin_old,
                cos_new, sin_new, apply_rope, (float*)k_out, (float*)v_out);
            break;
        default: return FADE_ERR_INVALID_ARG;
    }
    FADE_LAUNCH_CHECK();
    return FADE_OK;
}
