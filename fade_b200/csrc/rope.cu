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
    int64_t g = (n + 255) / 256;
    if (g > 148 * 16) g = 148 * 16;
    cudaStream_t st = as_stream(stream);
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
