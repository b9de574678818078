/*
 * fade_b200.h -- C ABI of libfade_sm100.so, the sm_100a (B200) implementation of
 * FADE's tiered KV-cache hot path.
 *
 * Every entry point:
 *   - is extern "C", takes plain pointers, sizes and strides (no torch types);
 *   - takes caller-owned device buffers and a cudaStream_t passed as void*;
 *   - allocates nothing and frees nothing (scratch space is the caller's
 *     `workspace`, sized by the matching *_workspace_size call);
 *   - returns an int status: FADE_OK (0) or one of fade_status below;
 *     fade_status_string() turns it into the message the Python layer raises.
 *
 * Reference interfaces replaced (paths inside the FADE project, fade-kv 1.1.0):
 *   fade/quant.py, fade/rotated_quant.py, fade/cache.py, fade/rope.py,
 *   fade/kernels/fused_int4_attn.py, fade/kernels/int4_attention.py.
 * The binding used by the Python package is fade_b200/_lib.py (ctypes).
 */
#ifndef FADE_B200_H
#define FADE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Status codes and element types                                             */
/* ------------------------------------------------------------------------ */
typedef enum fade_status {
    FADE_OK = 0,
    FADE_ERR_INVALID_ARG = 1,   /* null pointer, negative size, bad enum      */
    FADE_ERR_ODD_DIM = 2,       /* last dim not divisible by the pack factor  */
    FADE_ERR_GROUP = 3,         /* S not divisible by group_size              */
    FADE_ERR_UNSUPPORTED = 4,   /* shape/dtype combination not compiled       */
    FADE_ERR_ALIGN = 5,         /* pointer/stride violates a 16-byte rule     */
    FADE_ERR_WORKSPACE = 6,     /* workspace missing or too small             */
    FADE_ERR_CUDA = 7,          /* a CUDA runtime call failed                 */
    FADE_ERR_TIMEOUT = 8        /* a bounded device wait gave up (see below)  */
} fade_status;

typedef enum fade_dtype {
    FADE_F16 = 0,
    FADE_BF16 = 1,
    FADE_F32 = 2
} fade_dtype;

/* Strided 4-D view [B, H, S, D]; strides in ELEMENTS. */
typedef struct fade_view4 {
    int64_t B, H, S, D;
    int64_t sb, sh, ss, sd;
} fade_view4;

const char* fade_status_string(int status);
int fade_version(void);                      /* 100 * major + minor */
int fade_last_cuda_error(void);              /* cudaError_t of the last FADE_ERR_CUDA */
/* Makes `device` current for the library's CUDA runtime on the calling host
 * thread (the library links the runtime statically, so it keeps its own
 * notion of the current device).  Call before launching on that device. */
int fade_set_device(int device);
/* Number of SMs of the current device (148 on B200). */
int fade_sm_count(void);

/* ------------------------------------------------------------------------ */
/* K1: symmetric quantisation + bit packing (run on tier reassignment)        */
/* ------------------------------------------------------------------------ */

/* Replaces fade/quant.py:61-75 quant_k_int4 (+ _pack_int4_last_dim 26-43).
 * Per-channel INT4 over the S axis.  x: [B,H,S,D] (strided, F16/BF16).
 * packed: contiguous u8 [B,H,S,D/2], byte d = (q[2d]&15)<<4 | (q[2d+1]&15).
 * scale : contiguous [B,H,1,D] in x's dtype.  Bit-exact with the reference's
 * per-op rounding: scale = rnd(absmax/7), inv = rnd(rnd(1/absmax)*7),
 * q = clamp(rint(rnd(x*inv)), -8, 7).  D odd -> FADE_ERR_ODD_DIM. */
int fade_quant_int4_k(const void* x, int dtype, fade_view4 xv,
                      uint8_t* packed, void* scale, void* stream);

/* Replaces fade/quant.py:78-92 quant_v_int4: per-token INT4 (absmax over D).
 * scale: contiguous [B,H,S,1]. */
int fade_quant_int4_v(const void* x, int dtype, fade_view4 xv,
                      uint8_t* packed, void* scale, void* stream);

/* Replaces fade/quant.py:95-112 quant_k_int2 and 130-150 quant_v_int2 (same
 * arithmetic): groups of `group` tokens along S, per (group, channel) scale,
 * codes in [-2,1].  S % group != 0 -> FADE_ERR_GROUP.
 * codes_i8 (nullable): contiguous int8 [B,H,S,D] (the reference's storage).
 * codes_u8 (nullable): contiguous u8 [B,H,S,D/4], 4 codes per byte,
 *   byte = (c0&3)<<6 | (c1&3)<<4 | (c2&3)<<2 | (c3&3)  (fade/rotated_quant.py:35-48).
 * scale: contiguous [B,H,S/group,D] in x's dtype. */
int fade_quant_int2_grouped(const void* x, int dtype, fade_view4 xv, int group,
                            int8_t* codes_i8, uint8_t* codes_u8, void* scale,
                            void* stream);

/* Replaces fade/quant.py:26-58 and fade/rotated_quant.py:35-69 (pack/unpack).
 * rows x D codes, contiguous.  bits = 4 or 2. */
int fade_pack_codes(const int8_t* q, int64_t rows, int64_t D, int bits,
                    uint8_t* out, void* stream);
int fade_unpack_codes(const uint8_t* packed, int64_t rows, int64_t D, int bits,
                      int8_t* out, void* stream);

/* Replaces fade/quant.py:124-127 dequant_int4, 153-176 dequant_*_int2 and
 * 115-121 dequant: out = rnd(fp(q) * fp(scale)) in `dtype`.
 * codes: u8 packed rows of D*bits/8 bytes (bits 4 or 2) or int8 rows (bits 8).
 * scale_mode: 0 per-channel [B,H,1,D]; 1 per-token [B,H,S,1];
 *             2 grouped [B,H,S/group,D].  out: contiguous [B,H,S,D]. */
int fade_dequant(const void* codes, int bits, const void* scale, int scale_mode,
                 int group, int dtype, int64_t B, int64_t H, int64_t S, int64_t D,
                 void* out, void* stream);

/* Replaces fade/rotated_quant.py:106-131 rotated_quant_k (kind 0, per-channel
 * scale over S) and 148-173 rotated_quant_v (kind 1, per-token scale).
 * x_rot = x @ R^T in fp32, then symmetric quant at `bits` (2, 3 or 4) with
 * fp32 math; scale is cast to x's dtype.  bf16 x at D = 128 with 2- or 4-bit
 * codes, unit channel stride and 16-byte aligned rows and packed output:
 * tensor cores (R split exactly into three bf16 parts, fp32 accumulation in
 * the tensor core's order); otherwise CUDA cores with sequential-d
 * accumulation and no FMA contraction.  packed: bits 4 -> [..,D/2], 2 -> [..,D/4], 3 -> int8 [..,D].
 * R: [D,D] fp32 row-major on the device, 16-byte aligned (else FADE_ERR_ALIGN);
 * D a multiple of 4, at most 128.  workspace: >= B*H*D*4 bytes
 * (per-channel absmax, kind 0 only). */
int fade_rotated_quant(const void* x, int dtype, fade_view4 xv, const float* R,
                       int bits, int kind, uint8_t* packed, void* scale,
                       void* workspace, size_t ws_bytes, void* stream);

/* No counterpart in the reference (its rotation is a library matmul): reads
 * and clears the flag a tensor-core fade_rotated_quant kernel sets when its
 * bounded wait for its own MMAs gave up (the outputs of that call are then
 * undefined).  Synchronises `stream`.  FADE_OK or FADE_ERR_TIMEOUT. */
int fade_rotated_quant_check(void* stream);

/* Replaces fade/rotated_quant.py:134-145 / 176-187: out = rnd(rnd(q*scale) @ R)
 * (dequant in `dtype`, rotation in fp32).  scale_mode 0 (K) or 1 (V). */
int fade_rotated_dequant(const uint8_t* packed, int bits, const void* scale,
                         int scale_mode, const float* R, int dtype, int64_t B,
                         int64_t H, int64_t S, int64_t D, void* out, void* stream);

/* ------------------------------------------------------------------------ */
/* K3: eviction survivors -- gather + un-RoPE at old positions + re-RoPE at    */
/* new positions, one pass (replaces fade/cache.py:914-935 with               */
/* _inverse_rope 301-311 and _apply_rope 290-299).                              */
/* ------------------------------------------------------------------------ */
/* k_in, v_in: [B,H,S,D] strided (dtype).  keep_idx: int64 [n_kept] device
 * indices into S (ascending).  cos_old/sin_old: fp32 [S,D]; cos_new/sin_new:
 * fp32 [n_kept,D] (the RopeScheme tables, fade/rope.py:72-93).
 * k_out, v_out: contiguous [B,H,n_kept,D].  k_out = rnd(apply(rnd(inverse(k))))
 * with the reference's fp32 op order; v_out is a bit copy.  v_in/v_out may be
 * null.  apply_rope = 0 performs the gather only. */
int fade_rerope_gather(const void* k_in, const void* v_in, int dtype, fade_view4 kv,
                       const int64_t* keep_idx, int64_t n_kept,
                       const float* cos_old, const float* sin_old,
                       const float* cos_new, const float* sin_new, int apply_rope,
                       void* k_out, void* v_out, void* stream);

/* ------------------------------------------------------------------------ */
/* Age-out: the token leaving the FP16 recent window joins the INT4 middle.    */
/* (Extension beyond the reference, which re-quantises the whole middle;      */
/* K keeps its frozen per-channel scale, V gets its own per-token scale.)      */
/* ------------------------------------------------------------------------ */
/* Recent window = ring buffer ring_k/ring_v [B,H,ring_cap,D] (dtype, rows of D
 * contiguous; strides ring_sb, ring_sh in elements).  Middle = k_packed /
 * v_packed u8 rows of D/2 bytes, row (b,h,t) = b*mid_sb + h*mid_sh + t, with
 * v_scale (one dtype element per row) and the frozen per-channel K scale
 * k_scale [B,H,D].  mid_len: device int32 [B], tokens in the middle per row.
 * For each b, with n = mid_len[b] and slot = (n - ring_origin) mod ring_cap:
 *   for each h: the ring token (b,h,slot) is quantised into middle row
 *   (b,h,n):  K code = clamp(rint(fp32(x) / fp32(ks)), -8, 7) (0 where ks == 0),
 *             V exactly as fade_quant_int4_v on the single token;
 *   then, if k_new/v_new are given ([B,H,D], strides new_sb/new_sh), the new
 *   token is written into the freed ring slot;  finally mid_len[b] = n + 1.
 * Rows with n >= mid_cap are left untouched (mid_len is not advanced).
 * All positions come from device memory, so the call can be graph-captured. */
int fade_age_out_int4(void* ring_k, void* ring_v, int dtype,
                      int64_t B, int64_t H, int64_t D,
                      int64_t ring_cap, int64_t ring_sb, int64_t ring_sh, int64_t ring_origin,
                      uint8_t* k_packed, uint8_t* v_packed, void* v_scale,
                      const void* k_scale, int64_t mid_sb, int64_t mid_sh, int64_t mid_cap,
                      int32_t* mid_len,
                      const void* k_new, const void* v_new, int64_t new_sb, int64_t new_sh,
                      void* stream);

/* ------------------------------------------------------------------------ */
/* K2: fused tiered decode attention (replaces fade/cache.py:693-808          */
/* _materialize + the HF SDPA over it, and fade/kernels/fused_int4_attn.py     */
/* :277-342 fused_int4_sdpa).                                                   */
/* ------------------------------------------------------------------------ */
typedef enum fade_seg_kind {
    FADE_SEG_FP = 0,          /* dtype K/V rows of D elements (sink / recent)  */
    FADE_SEG_INT4 = 1,        /* INT4 K per-channel scale, INT4 V per-token    */
    FADE_SEG_INT4K_INT2V = 2, /* INT4 K per-channel, 2-bit V grouped per chan. */
    FADE_SEG_ROT = 3          /* rotated: K per-channel, V per-token, `bits`   */
} fade_seg_kind;

/* One tier of K/V for all (b, kv-head).  Token t of (b,h) lives at
 *   row = (row_base ? row_base[b*Hkv+h] : b*row_sb + h*row_sh) + t
 * in the K/V arrays (FP: rows of D dtype elements; quantised: rows of packed
 * bytes, D*bits/8 per row, 16-byte aligned, contiguous rows).
 * V per-token scales are indexed by the same row; grouped V scales by
 * row / group (rows must start on a group boundary).  K per-channel scales:
 * k_scale + (b*ks_sb + h*ks_sh) elements, D contiguous.
 * Token count: lens ? lens[b] : len (max_len bounds lens[]). */
typedef struct fade_kv_segment {
    int32_t kind;
    int32_t bits;            /* FADE_SEG_ROT: 2 or 4 */
    int32_t group;           /* FADE_SEG_INT4K_INT2V: tokens per V scale group */
    int32_t reserved;
    const void* k;
    const void* v;
    const void* k_scale;
    const void* v_scale;
    int64_t row_sb, row_sh;
    const int64_t* row_base;
    const int32_t* lens;     /* device int32 [B] or null                        */
    int64_t len;
    int64_t max_len;         /* bound on lens[] (sizes the grid)                */
    int64_t ks_sb, ks_sh;
    int64_t n_rows;          /* rows held by k/v (bounds the TMA reads); 0 = derive
                                from the dense strides (required with row_base or
                                page_table) */
    /* Paged middle (quantised tiers; FADE_PAGE_TOKENS-token pages): when
     * page_table is set, token t of (b,h) lives at row
     *   page_table[(b*Hkv+h)*pages_per_row + t/FADE_PAGE_TOKENS]*FADE_PAGE_TOKENS
     *   + t%FADE_PAGE_TOKENS
     * of a shared page pool (codes, per-token V scales; grouped V scales at
     * row/group) instead of row_base / row_sb / row_sh.  Device int32 table.
     * Not combined with fade_decode_attn_age_out (FADE_ERR_UNSUPPORTED).
     * (Block tables for continuous batching; the reference's roadmap item A1,
     * it has no paged layout itself.) */
    const int32_t* page_table;
    int64_t pages_per_row;
} fade_kv_segment;

#define FADE_PAGE_TOKENS 128

#define FADE_MAX_SEGMENTS 4

typedef struct fade_decode_desc {
    int32_t dtype;           /* q, out, FP tiers, scales: FADE_F16 / FADE_BF16 */
    int32_t B, Hq, Hkv, D;
    int32_t n_q;             /* query positions per head (1 = decode)          */
    float sm_scale;          /* softmax scale (1/sqrt(D) in the reference)     */
    const void* q;  int64_t q_sb, q_sh, q_ss;    /* [B,Hq,n_q,D], elements */
    void* out;      int64_t o_sb, o_sh, o_ss;
    const float* rotation;   /* [D,D] fp32, 16-byte aligned; required with a
                                FADE_SEG_ROT tier                               */
    int32_t n_segments;
    int32_t n_ctas;          /* 0 = auto (persistent grid: SMs x occupancy)    */
    const int32_t* cu_units; /* optional device int32 [B*Hkv+1]: prefix sum over
                                (b,h) of ceil(len/128) for the quantised tier
                                (ragged batches); null = every (b,h) gets
                                ceil(max_len/128) units, shorter rows skip
                                their empty units */
    fade_kv_segment seg[FADE_MAX_SEGMENTS];
} fade_decode_desc;

/* Bytes of zero-initialised workspace fade_decode_attn needs for `d`.  The
 * workspace carries split-K partials, an error word and the age-out
 * counters of fade_decode_attn_age_out (each returns to zero by the end of
 * every call); zero-fill it once when allocating it. */
size_t fade_decode_attn_workspace_size(const fade_decode_desc* d);

/* Attention of q over the union of all segments' tokens (order-free):
 * out = softmax(q K^T * sm_scale) V, GQA head hq -> kv head hq / (Hq/Hkv).
 * Quantised tiers are dequantised in registers; K/V never round-trip HBM. */
int fade_decode_attn(const fade_decode_desc* d, void* workspace, size_t ws_bytes,
                     void* stream);

/* One decode step of one layer: fade_age_out_int4 followed by
 * fade_decode_attn, fused (no counterpart in the reference, which keeps new
 * tokens in FP16 until its next reassignment, fade/cache.py:881-1057).
 * seg[ring_seg] is the FP recent-window ring (rows of D, row_sb / row_sh
 * strides, ring_cap rows per (b,h)); seg[mid_seg] the FADE_SEG_INT4 middle
 * with device lengths `lens` (= mid_len [B]) and capacity max_len.  For each b,
 * with n = lens[b] and slot = (n - ring_origin) mod ring_cap, when n < max_len
 * the result equals: quantise ring token `slot` into middle row n (K against
 * its frozen per-channel scale, V with its own per-token scale, exactly as
 * fade_age_out_int4), put k_new/v_new ([B,Hkv,D], strides new_sb / new_sh)
 * into the freed slot, lens[b] = n + 1, then attention over all tiers
 * (n_q must be 1).  Rows with n >= max_len are attended unchanged and the new
 * token is dropped, as fade_age_out_int4 does.
 * With prefetch_tiers = 1 the call may read the cache tiers (not q, k_new,
 * v_new) before the preceding kernel on the stream has finished: set it only
 * when that kernel does not write them.  The tiers include their device
 * lengths: the middle's `lens` (mid_len) and the ring's counts.  A preceding
 * fade_decode_attn_age_out or fade_age_out_int4 on the SAME layer writes
 * them, so two such calls on one layer back to back need prefetch_tiers = 0
 * (a chain over two or more layers may set it: each call then follows
 * another layer's). */
typedef struct fade_age_out_desc {
    int32_t ring_seg, mid_seg;
    int64_t ring_cap, ring_origin;
    const void* k_new;
    const void* v_new;
    int64_t new_sb, new_sh;          /* elements */
    int32_t prefetch_tiers;
    int32_t reserved;
} fade_age_out_desc;

int fade_decode_attn_age_out(const fade_decode_desc* d, const fade_age_out_desc* a,
                             void* workspace, size_t ws_bytes, void* stream);

/* No counterpart in the reference.  fade_decode_attn without a workspace
 * argument, for callers that cannot allocate device memory when they run
 * attention (a serving runtime handed a fixed memory pool, a plugin host that
 * forbids cudaMalloc after start-up, a caller with nowhere to keep a workspace
 * between calls).  Scratch space comes from one array compiled into the
 * library: fade_decode_attn_noalloc_max_bytes() bytes (32 MiB), reserved on
 * every GPU that loads the library until the process exits.  A call whose
 * fade_decode_attn_workspace_size() exceeds that returns FADE_ERR_WORKSPACE.
 * The first call on a device looks the array's device address up
 * (cudaGetSymbolAddress); make that first call before any stream capture.
 * All calls share the one array: calls that can overlap on the GPU (different
 * streams, or different host threads) race and must be serialised by the
 * caller.  Allocates nothing (no cudaMalloc / cudaFree). */
size_t fade_decode_attn_noalloc_max_bytes(void);
int fade_decode_attn_noalloc(const fade_decode_desc* d, void* stream);

/* Companion of fade_decode_attn_noalloc (no counterpart in the reference):
 * reads and clears the built-in array's device error word, as
 * fade_workspace_check does for a workspace (synchronises the stream).
 * Returns FADE_ERR_TIMEOUT when a bounded device wait of any earlier
 * fade_decode_attn_noalloc call on the current device gave up (that call's
 * output is not valid), FADE_OK otherwise.  The error word is sticky until
 * this call clears it. */
int fade_decode_attn_noalloc_check(void* stream);

/* Middle-kernel family for INT4 K and V at D = 128 (no counterpart in the
 * reference): 0 = mma.sync (default), 1 = tcgen05 (dequantised K in tensor
 * memory, V in shared memory, accumulators in tensor memory).  Both give
 * results within the same tolerance of the reference; process-wide, read
 * when a call builds its plan (plans already captured in a CUDA graph keep
 * their kernel).  Returns FADE_ERR_INVALID_ARG for other values. */
int fade_set_middle_kernel(int kind);
int fade_get_middle_kernel(void);

/* Reads and clears the device error word of a workspace (synchronises the
 * stream).  Returns FADE_OK or FADE_ERR_TIMEOUT. */
int fade_workspace_check(void* workspace, size_t ws_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* FADE_B200_H */
