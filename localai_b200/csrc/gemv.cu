// Decode GEMV / small-batch matmul over raw GGML block-quant rows (sm_100a).
//
// y[t, r] = sum_c W[r, c] * x[t, c] for W stored as the raw GGUF bytes of a
// [rows, cols] Q4_0/Q8_0/Q4_K/Q5_K/Q6_K matrix -- the computation of
// localai_*_matvec / localai_*_matmul in the reference
// (engine/native_quant.cpp:126-337 row kernels, :705-768 exports).
//
// Design (HBM-bound; ~0.56 B of weight per value for Q4_K):
// * One producer thread per CTA streams contiguous row tiles of the raw bytes
//   into a ring of shared-memory stages with non-tensor bulk copies
//   (cp.async.bulk, mbarrier complete_tx).  Any sub-16-byte tail is copied by
//   the producer with plain loads before it arrives on the stage barrier.
// * Consumer threads are "column stationary": a group of threads covers one
//   full row, each thread owning CPT fixed units (64 values of a K-quant
//   super-block, or one 32-value Q8_0/Q4_0 block); the activation values of
//   its units stay in registers for the whole kernel.  Groups take different
//   rows of a stage.  x is read once per CTA: quantised in the prologue into
//   shared memory (one 16-value task per thread at a time), then loaded into
//   the consumers' registers; after that the shared-memory traffic is the
//   weight stream and the per-stage partial sums.
// * Grouped mode (MoE experts at small batch): blockIdx.y selects a weight
//   matrix and a token range read from device offsets (validated in-kernel).
// * Integer dot products.  x is converted once per CTA to fixed point,
//   xq = rint(x / s) with s = max|x_unit| / (2^22 - 4) (|xq| < 2^22), held as
//   three byte planes (xq = 65536*b2 + 256*b1 + b0; b2 signed, b1/b0
//   unsigned).  The unpacked 4/5/6/8-bit quants are multiplied against the
//   planes with dp4a (4 products per instruction, exact int32 sums) and every
//   sub-block sum is scaled and accumulated in f32.  The activation grid step
//   is ~2^-22 of the unit's max |x| -- the order of f32 rounding -- so
//   results agree with the f32 dot product to f32-level accuracy (the
//   reference itself quantises x to int8 for Q4_K/Q5_K and int16 for Q6_K,
//   engine/native_quant.cpp:53-109).
// * Per-stage partial sums are reduced with warp shuffles, then across the
//   group's warps through shared memory in a fixed order (deterministic).
#include "common.cuh"
#include <algorithm>

namespace b200q {

struct GemvArgs {
    const uint8_t *w;
    const float *x;       // [tokens, cols]
    float *y;             // y[t * ys_t + r * ys_r]
    long long ys_t, ys_r;
    int rows, cols, tokens;
    int rb;               // bytes per row
    int units;            // units per row
    int nct;              // consumer threads per group (multiple of 32)
    int groups;           // row groups per CTA
    int stage_rows;       // groups * RPG
    int stage_bytes;      // bytes per shared stage buffer
    int stages;
    int *err;
    // grouped mode (grp_off != nullptr): blockIdx.y = group g, whose weights
    // start at w + g * w_group_stride and whose tokens are rows
    // [grp_off[g], grp_off[g+1]) of x and y (at most ``tokens`` of them)
    const int *grp_off;
    long long w_group_stride;
    int grp_rows;         // rows of x and y: every group's range must lie inside
    int n_groups;         // host side: grid.y
    int active_groups;    // host side: groups expected to hold tokens (sizes grid.x)
};

// Unit geometry per type: values per unit, units per block, x words per unit.
template <int T> struct Unit;
template <> struct Unit<T_Q4_K> { static constexpr int UV = 64, UPB = 4, NW = 16; };
template <> struct Unit<T_Q5_K> { static constexpr int UV = 64, UPB = 4, NW = 16; };
template <> struct Unit<T_Q6_K> { static constexpr int UV = 64, UPB = 4, NW = 16; };
template <> struct Unit<T_Q8_0> { static constexpr int UV = 32, UPB = 1, NW = 8; };
template <> struct Unit<T_Q4_0> { static constexpr int UV = 32, UPB = 1, NW = 8; };

// Activation slice of one unit in fixed point (three byte planes).
template <int NW>
struct XU {
    uint32_t b2[NW];    // signed top bytes of xq, 4 per word
    uint32_t b1[NW];    // unsigned middle bytes
    uint32_t b0[NW];    // unsigned low bytes
    float s;            // x ~= s * xq
    float sum[2];       // exact f32 sums of x over the two 32-value runs
    float qsum[4];      // sums of xq over the four 16-value runs (as f32)
};

// Sum of q*xq for one 32-value run from the three plane sums:
// 65536*a2 + 256*a1 + a0 (the two low planes combine exactly in int32).
__device__ __forceinline__ float planes_f(int a2, int a1, int a0)
{
    return fmaf((float)a2, 65536.0f, (float)(a1 * 256 + a0));
}

// Column of the first value of the two 32-value runs of unit u.
template <int T>
__device__ __forceinline__ void unit_cols(int u, int &c0, int &c1)
{
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        const int blk = u >> 2, p = u & 3;
        c0 = blk * 256 + 64 * p;
        c1 = c0 + 32;
    } else if constexpr (T == T_Q6_K) {
        const int blk = u >> 2, h = (u >> 1) & 1, a = u & 1;
        c0 = blk * 256 + 128 * h + 32 * a;
        c1 = c0 + 64;
    } else {
        c0 = u * 32;
        c1 = c0;
    }
}

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c)   // u8 x s8
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c)   // u8 x u8
{
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c)   // s8 x s8
{
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c)   // s8 x u8
{
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 32 bytes from a shared address that is at least 2-byte aligned.
__device__ __forceinline__ void lds256_any(uint32_t a, uint32_t o[8])
{
    const uint32_t base = a & ~3u, sh = (a & 3u) * 8u;
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = lds32(base + 4 * i);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __funnelshift_r(w[i], w[i + 1], sh);
}
__device__ __forceinline__ void lds128x2(uint32_t a, uint32_t o[8], bool aligned16)
{
    if (aligned16) {
        const uint4 v0 = lds128(a), v1 = lds128(a + 16);
        o[0] = v0.x; o[1] = v0.y; o[2] = v0.z; o[3] = v0.w;
        o[4] = v1.x; o[5] = v1.y; o[6] = v1.z; o[7] = v1.w;
    } else {
        lds256_any(a, o);
    }
}

__device__ __forceinline__ float ubyte_f(uint32_t v, int k) { return (float)((v >> (8 * k)) & 0xffu); }

// ---------------------------------------------------------------- unit dots
// Each adds the unit's contribution for NTOK tokens into acc[].
// blk: shared address of the block start; p: unit index inside the block.

// Accumulate one 4-byte word of unsigned quants against word k of the planes.
#define B200Q_DOT_U(Q, XX, K, A2, A1, A0)       \
    A2 = dp4a_us((Q), (XX).b2[K], A2);          \
    A1 = dp4a_uu((Q), (XX).b1[K], A1);          \
    A0 = dp4a_uu((Q), (XX).b0[K], A0);

template <int NTOK, bool AL>
__device__ __forceinline__ void dot_q4k(uint32_t blk, int p, const XU<16> (&X)[NTOK], float (&acc)[NTOK])
{
    const uint4 hdr = lds128_any<AL>(blk);
    uint32_t w[8];
    lds128x2(blk + 16 + 32 * p, w, AL);
    const uint32_t sp = k_scales_packed(hdr, p);
    const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
    const float sc0 = ubyte_f(sp, 0), sc1 = ubyte_f(sp, 1), mn0 = ubyte_f(sp, 2), mn1 = ubyte_f(sp, 3);
    int a[NTOK][6];
#pragma unroll
    for (int t = 0; t < NTOK; ++t)
#pragma unroll
        for (int i = 0; i < 6; ++i) a[t][i] = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t L = w[k] & 0x0F0F0F0Fu, H = (w[k] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int t = 0; t < NTOK; ++t) {
            B200Q_DOT_U(L, X[t], k, a[t][0], a[t][1], a[t][2]);
            B200Q_DOT_U(H, X[t], 8 + k, a[t][3], a[t][4], a[t][5]);
        }
    }
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
        const float i0 = planes_f(a[t][0], a[t][1], a[t][2]);
        const float i1 = planes_f(a[t][3], a[t][4], a[t][5]);
        acc[t] += (d * X[t].s) * fmaf(sc0, i0, sc1 * i1) - dmin * fmaf(mn0, X[t].sum[0], mn1 * X[t].sum[1]);
    }
}

template <int NTOK, bool AL>
__device__ __forceinline__ void dot_q5k(uint32_t blk, int p, const XU<16> (&X)[NTOK], float (&acc)[NTOK])
{
    const uint4 hdr = lds128_any<AL>(blk);
    uint32_t w[8], h[8];
    lds128x2(blk + 16, h, AL);
    lds128x2(blk + 48 + 32 * p, w, AL);
    const uint32_t sp = k_scales_packed(hdr, p);
    const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
    const float sc0 = ubyte_f(sp, 0), sc1 = ubyte_f(sp, 1), mn0 = ubyte_f(sp, 2), mn1 = ubyte_f(sp, 3);
    const int k0 = 2 * p;
    int a[NTOK][6];
#pragma unroll
    for (int t = 0; t < NTOK; ++t)
#pragma unroll
        for (int i = 0; i < 6; ++i) a[t][i] = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t L = (w[k] & 0x0F0F0F0Fu) | (((h[k] >> k0) & 0x01010101u) << 4);
        const uint32_t H = ((w[k] >> 4) & 0x0F0F0F0Fu) | (((h[k] >> (k0 + 1)) & 0x01010101u) << 4);
#pragma unroll
        for (int t = 0; t < NTOK; ++t) {
            B200Q_DOT_U(L, X[t], k, a[t][0], a[t][1], a[t][2]);
            B200Q_DOT_U(H, X[t], 8 + k, a[t][3], a[t][4], a[t][5]);
        }
    }
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
        const float i0 = planes_f(a[t][0], a[t][1], a[t][2]);
        const float i1 = planes_f(a[t][3], a[t][4], a[t][5]);
        acc[t] += (d * X[t].s) * fmaf(sc0, i0, sc1 * i1) - dmin * fmaf(mn0, X[t].sum[0], mn1 * X[t].sum[1]);
    }
}

template <int NTOK>
__device__ __forceinline__ void dot_q6k(uint32_t blk, int u, const XU<16> (&X)[NTOK], float (&acc)[NTOK])
{
    const int h = (u >> 1) & 1, a = u & 1;
    uint32_t ql[8], qh[8];
    lds256_any(blk + 64 * h + 32 * a, ql);
    lds256_any(blk + 128 + 32 * h, qh);
    const uint32_t sb = blk + 192 + 8 * h + 2 * a;
    const uint32_t s01 = lds_u16(sb), s45 = lds_u16(sb + 4);
    const float sc[4] = {(float)(int8_t)(s01 & 0xff), (float)(int8_t)(s01 >> 8), (float)(int8_t)(s45 & 0xff),
                         (float)(int8_t)(s45 >> 8)};
    const float d = h2f(lds_u16(blk + 208));
    const int shl = 4 - 2 * a, shr = 2 * a;
    int acc3[NTOK][4][3];
#pragma unroll
    for (int t = 0; t < NTOK; ++t)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc3[t][r][0] = acc3[t][r][1] = acc3[t][r][2] = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t L = (ql[k] & 0x0F0F0F0Fu) | ((qh[k] << shl) & 0x30303030u);
        const uint32_t H = ((ql[k] >> 4) & 0x0F0F0F0Fu) | ((qh[k] >> shr) & 0x30303030u);
        const int r0 = k >> 2, r1 = 2 + (k >> 2);
#pragma unroll
        for (int t = 0; t < NTOK; ++t) {
            B200Q_DOT_U(L, X[t], k, acc3[t][r0][0], acc3[t][r0][1], acc3[t][r0][2]);
            B200Q_DOT_U(H, X[t], 8 + k, acc3[t][r1][0], acc3[t][r1][1], acc3[t][r1][2]);
        }
    }
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < 4; ++r)   // sum (q-32)*xq over a 16-value run
            v = fmaf(sc[r], fmaf(-32.0f, X[t].qsum[r], planes_f(acc3[t][r][0], acc3[t][r][1], acc3[t][r][2])), v);
        acc[t] = fmaf(d * X[t].s, v, acc[t]);
    }
}

template <int NTOK>
__device__ __forceinline__ void dot_q8_0(uint32_t blk, const XU<8> (&X)[NTOK], float (&acc)[NTOK])
{
    const float d = h2f(lds_u16(blk));
    uint32_t q[8];
    lds256_any(blk + 2, q);
    int a2[NTOK], a1[NTOK], a0[NTOK];
#pragma unroll
    for (int t = 0; t < NTOK; ++t) a2[t] = a1[t] = a0[t] = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k)
#pragma unroll
        for (int t = 0; t < NTOK; ++t) {
            a2[t] = dp4a_ss(q[k], X[t].b2[k], a2[t]);
            a1[t] = dp4a_su(q[k], X[t].b1[k], a1[t]);
            a0[t] = dp4a_su(q[k], X[t].b0[k], a0[t]);
        }
#pragma unroll
    for (int t = 0; t < NTOK; ++t) acc[t] = fmaf(d * X[t].s, planes_f(a2[t], a1[t], a0[t]), acc[t]);
}

template <int NTOK>
__device__ __forceinline__ void dot_q4_0(uint32_t blk, const XU<8> (&X)[NTOK], float (&acc)[NTOK])
{
    const float d = h2f(lds_u16(blk));
    const uint4 q4 = lds128_any<false>(blk + 2);
    const uint32_t w[4] = {q4.x, q4.y, q4.z, q4.w};
    int a2[NTOK], a1[NTOK], a0[NTOK];
#pragma unroll
    for (int t = 0; t < NTOK; ++t) a2[t] = a1[t] = a0[t] = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t L = w[k] & 0x0F0F0F0Fu, H = (w[k] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int t = 0; t < NTOK; ++t) {
            B200Q_DOT_U(L, X[t], k, a2[t], a1[t], a0[t]);
            B200Q_DOT_U(H, X[t], 4 + k, a2[t], a1[t], a0[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
        const float qs = X[t].qsum[0] + X[t].qsum[1];
        acc[t] = fmaf(d * X[t].s, fmaf(-8.0f, qs, planes_f(a2[t], a1[t], a0[t])), acc[t]);
    }
}

template <int T, int NTOK, bool AL>
__device__ __forceinline__ void unit_dot(uint32_t blk, int c, const XU<Unit<T>::NW> (&X)[NTOK], float (&acc)[NTOK])
{
    if constexpr (T == T_Q4_K) dot_q4k<NTOK, AL>(blk, c, X, acc);
    else if constexpr (T == T_Q5_K) dot_q5k<NTOK, AL>(blk, c, X, acc);
    else if constexpr (T == T_Q6_K) dot_q6k<NTOK>(blk, c, X, acc);
    else if constexpr (T == T_Q8_0) dot_q8_0<NTOK>(blk, X, acc);
    else dot_q4_0<NTOK>(blk, X, acc);
}

// Packed activation of one (token, unit): the XU fields laid out as
// 3*NW plane words, then s, sum[2], qsum[4], padded to a multiple of 4 words.
template <int NW> struct XPackWords { static constexpr int N = ((3 * NW + 7) + 3) / 4 * 4; };

// One quantisation task covers 16 consecutive values of one (token, unit):
// words 4j .. 4j+3 (j = task % L, L = NW / 4 lanes per unit) of unit task / L.
// The L lanes of a unit are consecutive, so the unit's max |x| takes log2(L)
// shuffles and the 32-value sums one; the 16-value sums of xq stay inside the
// thread.  Quantisation: xq = rint(x * inv), inv = (2^22 - 4) / max|x| (so
// |xq| < 2^22 and the rounding is one FMA with the 1.5 * 2^23 magic constant),
// reconstructed with s = max|x| / (2^22 - 4); the two agree to f32 rounding.
constexpr float XQ_RANGE = 4194300.0f;          // 2^22 - 4
constexpr float XQ_MAGIC = 12582912.0f;         // 1.5 * 2^23
constexpr int XQ_MAGIC_BITS = 0x4B400000;

// Columns of x that quantisation task ``task`` reads (16 of them, from the
// returned pointer on): row t of x, words 4j .. 4j+3 of unit u.  With one
// token the unit index needs no division.
template <int T>
__device__ __forceinline__ const float *quantize_x_addr(const float *__restrict__ x, int cols, int units, int ntok,
                                                        int task)
{
    constexpr int L = Unit<T>::NW / 4;
    const int j = task % L, tu = task / L;
    const int u = ntok == 1 ? tu : tu % units, t = ntok == 1 ? 0 : tu / units;
    int c0 = 0, c1 = 0;
    unit_cols<T>(u, c0, c1);
    const int k = 4 * j;                                          // first word of the task
    return x + (long long)t * cols + (k < 8 ? c0 : c1) + 4 * (k & 7);
}

// Quantise one task's 16 values v[] and store its words (every lane of the
// warp must call this: the unit max and the 32-value sums use shuffles;
// ``valid`` masks the stores).
template <int T>
__device__ __forceinline__ void quantize_x_task16(const float4 (&v)[4], bool valid, int task, uint32_t xs)
{
    constexpr int NW = Unit<T>::NW, N = XPackWords<NW>::N, L = NW / 4;
    const int j = task % L, tu = task / L;
    float m = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w)
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v[w].x), fabsf(v[w].y)), fmaxf(fabsf(v[w].z), fabsf(v[w].w))));
#pragma unroll
    for (int o = 1; o < L; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const float inv = m > 0.f ? __frcp_rn(m) * XQ_RANGE : 0.f;
    uint32_t p2[4], p1[4], p0[4];
    int qs = 0;
    float sm = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const float e[4] = {v[w].x, v[w].y, v[w].z, v[w].w};
        uint32_t q[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            q[c] = (uint32_t)(__float_as_int(fmaf(e[c], inv, XQ_MAGIC)) - XQ_MAGIC_BITS);   // rint(e * inv)
            qs += (int)q[c];
        }
        sm += (e[0] + e[1]) + (e[2] + e[3]);
        // byte b of the four values -> one word per plane (two's complement:
        // q = 65536 * (int8)b2 + 256 * b1 + b0)
#pragma unroll
        for (int b = 0; b < 3; ++b) {
            const uint32_t sel = (uint32_t)b | ((4u + b) << 4);
            const uint32_t word = __byte_perm(__byte_perm(q[0], q[1], sel), __byte_perm(q[2], q[3], sel), 0x5410);
            (b == 2 ? p2 : b == 1 ? p1 : p0)[w] = word;
        }
    }
    sm += __shfl_xor_sync(0xffffffffu, sm, 1);       // the two tasks of a 32-value run
    if (valid) {
        const uint32_t o = xs + (uint32_t)tu * N * 4;
        const uint32_t k = 4u * j;
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(o + 4 * k), "r"(p2[0]), "r"(p2[1]), "r"(p2[2]), "r"(p2[3]) : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(o + 4 * (NW + k)), "r"(p1[0]), "r"(p1[1]), "r"(p1[2]), "r"(p1[3]) : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(o + 4 * (2 * NW + k)), "r"(p0[0]), "r"(p0[1]), "r"(p0[2]), "r"(p0[3]) : "memory");
        if (j == 0)
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(o + 4 * (3 * NW)), "r"(__float_as_uint(m * (1.0f / XQ_RANGE))) : "memory");
        if ((j & 1) == 0)
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(o + 4 * (3 * NW + 1 + (j >> 1))), "r"(__float_as_uint(sm)) : "memory");
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(o + 4 * (3 * NW + 3 + j)), "r"(__float_as_uint((float)qs)) : "memory");
    }
}

// Cooperative quantisation of x [ntok, cols] into packed per-unit words in
// shared memory (xs[(t * units + u) * N ...]); every lane of the calling warps
// must execute this.  A thread's tasks are taken in batches of MAXIT whose
// loads are all issued before any is used (one L2 round trip per batch).
template <int T>
__device__ __forceinline__ void quantize_x_smem(const float *__restrict__ x, int cols, int units, int ntok, uint32_t xs,
                                                int tid, int nthreads)
{
    constexpr int L = Unit<T>::NW / 4;
    constexpr int MAXIT = 4;
    const int tasks = ntok * units * L;
    const int iters = (tasks + nthreads - 1) / nthreads;
    for (int i0 = 0; i0 < iters; i0 += MAXIT) {
        float4 f[MAXIT][4];
#pragma unroll
        for (int i = 0; i < MAXIT; ++i) {
            const int task = (i0 + i) * nthreads + tid;
            if (i0 + i < iters && task < tasks) {
                const float4 *p = reinterpret_cast<const float4 *>(quantize_x_addr<T>(x, cols, units, ntok, task));
#pragma unroll
                for (int w = 0; w < 4; ++w) f[i][w] = __ldg(p + w);
            } else {
#pragma unroll
                for (int w = 0; w < 4; ++w) f[i][w] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
#pragma unroll
        for (int i = 0; i < MAXIT; ++i) {
            const int task = (i0 + i) * nthreads + tid;
            if (i0 + i < iters) quantize_x_task16<T>(f[i], task < tasks, task, xs);   // warp-uniform condition
        }
    }
}

// Load one unit's packed activation from shared memory.
template <int T>
__device__ __forceinline__ void load_unit_x(uint32_t xsu, bool valid, XU<Unit<T>::NW> &X)
{
    constexpr int NW = Unit<T>::NW, N = XPackWords<NW>::N;
    uint32_t w[N];
#pragma unroll
    for (int k = 0; k < N / 4; ++k) {
        const uint4 v = valid ? lds128(xsu + 16 * k) : make_uint4(0, 0, 0, 0);
        w[4 * k] = v.x; w[4 * k + 1] = v.y; w[4 * k + 2] = v.z; w[4 * k + 3] = v.w;
    }
#pragma unroll
    for (int k = 0; k < NW; ++k) {
        X.b2[k] = w[k];
        X.b1[k] = w[NW + k];
        X.b0[k] = w[2 * NW + k];
    }
    X.s = __uint_as_float(w[3 * NW]);
    X.sum[0] = __uint_as_float(w[3 * NW + 1]);
    X.sum[1] = __uint_as_float(w[3 * NW + 2]);
#pragma unroll
    for (int r = 0; r < 4; ++r) X.qsum[r] = __uint_as_float(w[3 * NW + 3 + r]);
}

// ---------------------------------------------------------------- kernel
// Shared layout: [full mbarriers][empty mbarriers] (128 B) | per-stage
// partial-sum slots | quantised activations | stage buffers (128-B aligned).
//
// Roles.  Consumer warps: wait for a stage, add their units' dot products
// for each of their rows, reduce the per-row values across the warp with a
// butterfly (each lane ends with one finished row value), store them in the
// stage's partial-sum slot and arrive on the stage's "empty" barrier.  The
// producer warp: once a stage is empty it sums the per-warp partials of every
// row in a fixed order, writes y, and refills the stage with the next row
// tile.  Consumers never wait on each other.

// Thread cap per configuration so that the stationary x registers fit.
template <int CPT, int NTOK>
struct GemvCap { static constexpr int THREADS = (CPT * NTOK >= 4) ? 256 : 384; };

// Butterfly transpose-reduction of V values per lane (V a power of two <= 32):
// afterwards every lane holds the warp-wide sum of value (lane >> (5 - log2 V)).
template <int V>
__device__ __forceinline__ float warp_transpose_reduce(float (&v)[V], int lane)
{
    int n = V;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (n > 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                if (i < n / 2) {
                    const float send = up ? v[i] : v[i + n / 2];
                    const float keep = up ? v[i + n / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            n >>= 1;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    return v[0];
}

template <int T, int CPT, int NTOK, int RPG, bool AL>
__global__ void __launch_bounds__(GemvCap<CPT, NTOK>::THREADS) gemv_kernel(const GemvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int BYTES = Fmt<T>::BYTES;
    constexpr int V = RPG * NTOK;                                 // values per lane per pass
    constexpr int LOGV = V == 1 ? 0 : V == 2 ? 1 : V == 4 ? 2 : V == 8 ? 3 : 4;
    const int tid = threadIdx.x;
    const int ncons = a.groups * a.nct;
    const int nwarps_c = ncons >> 5;
    const int nwg = a.nct >> 5;                                   // warps per group
    const uint8_t *wsrc = a.w;
    const float *xsrc = a.x;
    float *ydst = a.y;
    int tokens = a.tokens;
    if (a.grp_off) {
        // which experts run, and on how many tokens, comes from the previous kernel
        pdl_wait();
        const int t0 = a.grp_off[blockIdx.y], t1 = a.grp_off[blockIdx.y + 1];
        if (t0 < 0 || t1 < t0 || t1 > a.grp_rows || t1 - t0 > a.tokens) {      // offsets not usable: touch nothing
            if (threadIdx.x == 0) atomicExch(a.err, ERR_BAD_INDEX);
            pdl_launch_dependents();
            return;
        }
        tokens = t1 - t0;
        if (tokens == 0) {
            pdl_launch_dependents();
            return;
        }
        wsrc += (long long)blockIdx.y * a.w_group_stride;
        xsrc += (long long)t0 * a.cols;
        ydst += (long long)t0 * a.ys_t;
    }
    const int npass = (tokens + NTOK - 1) / NTOK;
    const int npass_max = (a.tokens + NTOK - 1) / NTOK;           // shared layout is sized for a.tokens
    const int slot_floats = npass_max * nwarps_c * V;             // partials of one stage
    const uint32_t sbase = smem_addr(smem);
    const uint32_t full0 = sbase, empty0 = sbase + 8 * a.stages;
    float *red = reinterpret_cast<float *>(smem + 128);
    constexpr int NWX = Unit<T>::NW, NX = XPackWords<NWX>::N;
    const uint32_t xbuf = (sbase + 128 + (uint32_t)a.stages * slot_floats * 4 + 15) & ~15u;
    const uint32_t stage0 = (xbuf + (uint32_t)(a.tokens * a.units * NX * 4) + 127) & ~127u;

    const long long r_begin = (long long)blockIdx.x * a.rows / gridDim.x;
    const long long r_end = (long long)(blockIdx.x + 1) * a.rows / gridDim.x;
    const int n_it = (int)((r_end - r_begin + a.stage_rows - 1) / a.stage_rows);

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, nwarps_c);
        }
        mbar_fence_init();
    }
    __syncthreads();
    // Weights are read-only for the whole stream, so the weight stream starts
    // before the dependency wait; x and y are touched only after pdl_wait().
    pdl_launch_dependents();

    if (tid >= ncons) {                        // ---- producer / reducer warp
        const int lane = tid - ncons;
        const uint64_t pol = policy_evict_first();
        bool ok = true;
        int issued = 0;
        for (int it = 0; it < n_it + a.stages && ok; ++it) {
            const int s = it % a.stages;
            if (it >= a.stages) {              // stage j = it - S is consumed: reduce it
                const int j = it - a.stages;
                if (j == 0) pdl_wait();
                if (!mbar_wait(empty0 + 8 * s, (j / a.stages) & 1, a.err)) { ok = false; break; }
                const long long row0 = r_begin + (long long)j * a.stage_rows;
                const int nr = (int)min((long long)a.stage_rows, r_end - row0);
                const float *slot = red + s * slot_floats;
                // value index: ((pass * groups + g) * V + rr * NTOK + t); warp partials
                // of group g live at slot[(pass * nwarps_c + g * nwg + wig) * V + vi].
                const int total = npass * a.groups * V;
                for (int idx = lane; idx < total; idx += 32) {
                    const int vi = idx % V, pg = idx / V;
                    const int g = pg % a.groups, pass = pg / a.groups;
                    const int rr = vi / NTOK, t = vi % NTOK;
                    const int lr = g + rr * a.groups, tok = pass * NTOK + t;
                    if (lr < nr && tok < tokens) {
                        const float *pp = slot + (pass * nwarps_c + g * nwg) * V + vi;
                        float v = 0.f;
                        for (int w = 0; w < nwg; ++w) v += pp[w * V];
                        ydst[tok * a.ys_t + (row0 + lr) * a.ys_r] = v;
                    }
                }
                __syncwarp();
            }
            if (it < n_it && lane == 0) {
                const long long row0 = r_begin + (long long)it * a.stage_rows;
                const int nr = (int)min((long long)a.stage_rows, r_end - row0);
                const uint8_t *gs = wsrc + row0 * a.rb;
                const uint8_t *ge = gs + (long long)nr * a.rb;
                const uint8_t *a0 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(gs) & ~(uintptr_t)15);
                const uint8_t *a1 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(ge) & ~(uintptr_t)15);
                const uint32_t dst = stage0 + (uint32_t)s * a.stage_bytes;
                for (const uint8_t *p = a1; p < ge; ++p)           // < 16 tail bytes
                    asm volatile("st.shared.u8 [%0], %1;" ::"r"(dst + (uint32_t)(p - a0)), "h"((unsigned short)__ldg(p)));
                const uint32_t nbytes = (uint32_t)(a1 - a0);
                if (nbytes) {
                    mbar_arrive_expect_tx(full0 + 8 * s, nbytes);
                    bulk_g2s(dst, a0, nbytes, full0 + 8 * s, pol);
                } else {
                    mbar_arrive(full0 + 8 * s);
                }
                issued = it + 1;
            }
            __syncwarp();
        }
        if (!ok && lane == 0) {                // drain copies that may still be in flight
            for (int j = max(0, issued - a.stages); j < issued; ++j)
                mbar_wait(full0 + 8 * (j % a.stages), (j / a.stages) & 1, a.err);
        }
        return;
    }

    // ---- consumers
    constexpr int UPB = Unit<T>::UPB, NW = Unit<T>::NW;
    const int g = tid / a.nct, lt = tid % a.nct;
    const int wig = lt >> 5, lane = tid & 31;
    const int cw = g * nwg + wig;                                  // consumer warp index
    int uoff[CPT], uc[CPT], uidx[CPT];
    bool uval[CPT];
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
        const int u = lt + i * a.nct;
        uval[i] = u < a.units;
        uidx[i] = uval[i] ? u : 0;
        uoff[i] = (uidx[i] / UPB) * BYTES;
        uc[i] = uidx[i] % UPB;
    }
    XU<NW> X[CPT][NTOK];
    pdl_wait();                                          // x may come from the previous kernel
    quantize_x_smem<T>(xsrc, a.cols, a.units, tokens, xbuf, tid, ncons);
    named_bar_sync(1, ncons);
    auto load_x = [&](int pass) {
#pragma unroll
        for (int i = 0; i < CPT; ++i)
#pragma unroll
            for (int t = 0; t < NTOK; ++t) {
                const int tok = pass * NTOK + t;
                const bool v = uval[i] && tok < tokens;
                load_unit_x<T>(xbuf + (uint32_t)(((v ? tok : 0) * a.units + uidx[i]) * NX * 4), v, X[i][t]);
            }
    };
    if (npass == 1) load_x(0);

    for (int it = 0; it < n_it; ++it) {
        const int s = it % a.stages;
        if (!mbar_wait(full0 + 8 * s, (it / a.stages) & 1, a.err)) return;
        const long long row0 = r_begin + (long long)it * a.stage_rows;
        const int nr = (int)min((long long)a.stage_rows, r_end - row0);
        const uintptr_t gs = reinterpret_cast<uintptr_t>(wsrc + row0 * a.rb);
        const uint32_t base = stage0 + (uint32_t)s * a.stage_bytes + (uint32_t)(gs & 15);
        float *slot = red + s * slot_floats;
        for (int pass = 0; pass < npass; ++pass) {
            if (npass > 1) load_x(pass);
            float acc[RPG][NTOK];
#pragma unroll
            for (int rr = 0; rr < RPG; ++rr)
#pragma unroll
                for (int t = 0; t < NTOK; ++t) acc[rr][t] = 0.f;
            if (g + (RPG - 1) * a.groups < nr) {                  // full stage: no row checks
#pragma unroll
                for (int rr = 0; rr < RPG; ++rr) {
                    const uint32_t rbase = base + (uint32_t)((g + rr * a.groups) * a.rb);
#pragma unroll
                    for (int i = 0; i < CPT; ++i)
                        if (uval[i]) unit_dot<T, NTOK, AL>(rbase + uoff[i], uc[i], X[i], acc[rr]);
                }
            } else {
#pragma unroll
                for (int rr = 0; rr < RPG; ++rr) {
                    const int lr = g + rr * a.groups;
                    if (lr < nr) {
                        const uint32_t rbase = base + (uint32_t)(lr * a.rb);
#pragma unroll
                        for (int i = 0; i < CPT; ++i)
                            if (uval[i]) unit_dot<T, NTOK, AL>(rbase + uoff[i], uc[i], X[i], acc[rr]);
                    }
                }
            }
            float v[V];
#pragma unroll
            for (int rr = 0; rr < RPG; ++rr)
#pragma unroll
                for (int t = 0; t < NTOK; ++t) v[rr * NTOK + t] = acc[rr][t];
            const float r = warp_transpose_reduce<V>(v, lane);
            if ((lane & ((32 >> LOGV) - 1)) == 0) slot[(pass * nwarps_c + cw) * V + (lane >> (5 - LOGV))] = r;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty0 + 8 * s);
    }
}

// ---------------------------------------------------------------- host side
// Tuning knobs (defaults chosen on B200): target bytes of weights per stage
// and number of stages.
static int g_stage_target = 48 * 1024;
static int g_stages = 3;
static int g_rpg_max = 4;
static int g_ctas_per_sm = 0;     // 0 = as many as fit
static bool g_use_mma = true;     // batch-1 Q4_K on the integer tensor cores
void gemv_set_mma(bool on) { g_use_mma = on; }
void gemv_set_tuning(int stage_target_bytes, int stages, int rpg_max, int ctas_per_sm)
{
    if (stage_target_bytes > 0) g_stage_target = stage_target_bytes;
    if (stages > 0) g_stages = stages;
    if (rpg_max > 0) g_rpg_max = rpg_max;
    if (ctas_per_sm >= 0) g_ctas_per_sm = ctas_per_sm;
}

template <int T, int CPT, int NTOK, int RPG, bool AL>
static cudaError_t run_cfg(GemvArgs a, int threads, size_t smem, int num_sms, cudaStream_t st)
{
    auto kern = gemv_kernel<T, CPT, NTOK, RPG, AL>;
    // Attribute/occupancy queries are cached per instantiation (host calls
    // are serialised by the library's lock).
    static size_t attr_smem = 0;
    static int occ_threads = -1;
    static size_t occ_smem = 0;
    static int occ_per_sm = 0;
    cudaError_t e;
    if (smem > attr_smem) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        attr_smem = smem;
    }
    if (threads != occ_threads || smem != occ_smem) {
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ_per_sm, kern, threads, smem);
        if (e != cudaSuccess) return e;
        occ_threads = threads;
        occ_smem = smem;
    }
    int per_sm = occ_per_sm;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    if (g_ctas_per_sm > 0 && per_sm > g_ctas_per_sm) per_sm = g_ctas_per_sm;
    const long long tiles = (a.rows + a.stage_rows - 1) / a.stage_rows;
    long long grid = (long long)num_sms * per_sm;
    if (a.grp_off) grid = (grid + a.active_groups - 1) / a.active_groups;
    if (grid > tiles) grid = tiles;
    return launch_pdl(kern, dim3((unsigned)grid, a.grp_off ? (unsigned)a.n_groups : 1u), dim3(threads), smem, st, a);
}

template <int T, int CPT, int NTOK, int RPG>
static cudaError_t run_al(GemvArgs a, int threads, size_t smem, int num_sms, cudaStream_t st, bool al)
{
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        if (al) return run_cfg<T, CPT, NTOK, RPG, true>(a, threads, smem, num_sms, st);
    }
    return run_cfg<T, CPT, NTOK, RPG, false>(a, threads, smem, num_sms, st);
}

template <int T, int CPT, int NTOK>
static cudaError_t run_rpg(GemvArgs a, int rpg, int threads, size_t smem, int num_sms, cudaStream_t st, bool al)
{
    if constexpr (CPT * NTOK == 1) {
        switch (rpg) {
        case 1: return run_al<T, CPT, NTOK, 1>(a, threads, smem, num_sms, st, al);
        case 2: return run_al<T, CPT, NTOK, 2>(a, threads, smem, num_sms, st, al);
        default: return run_al<T, CPT, NTOK, 4>(a, threads, smem, num_sms, st, al);
        }
    }
    return run_al<T, CPT, NTOK, 1>(a, threads, smem, num_sms, st, al);
}

template <int T>
static cudaError_t run_type(GemvArgs a, int cpt, int ntok, int rpg, int threads, size_t smem, int num_sms,
                            cudaStream_t st, bool al)
{
    if (cpt == 1 && ntok == 1) return run_rpg<T, 1, 1>(a, rpg, threads, smem, num_sms, st, al);
    if (cpt == 1 && ntok == 2) return run_rpg<T, 1, 2>(a, rpg, threads, smem, num_sms, st, al);
    if (cpt == 1 && ntok == 4) return run_rpg<T, 1, 4>(a, rpg, threads, smem, num_sms, st, al);
    if (cpt == 2 && ntok == 1) return run_rpg<T, 2, 1>(a, rpg, threads, smem, num_sms, st, al);
    if (cpt == 2 && ntok == 2) return run_rpg<T, 2, 2>(a, rpg, threads, smem, num_sms, st, al);
    return run_rpg<T, 4, 1>(a, rpg, threads, smem, num_sms, st, al);
}

// One launch over tokens [0, tokens) of the given x/y.
static cudaError_t launch_gemv_chunk(int type, const void *w, const float *x, float *y, long long ys_t, long long ys_r,
                                     int rows, int cols, int tokens, int *err, int num_sms, cudaStream_t st,
                                     const int *grp_off = nullptr, long long w_group_stride = 0, int n_groups = 0,
                                     int active_groups = 1, long long row_stride = 0, int grp_rows = 0)
{
    const int vals = type_vals(type), bytes = type_bytes(type);
    const int upb = (vals == 256) ? 4 : 1;     // 64-value units in a K-quant block
    const int units = (cols / vals) * upb;
    const int nx = (vals == 256) ? XPackWords<16>::N : XPackWords<8>::N;
    // Smallest units-per-thread (CPT) whose group fits the thread cap of its
    // register budget; NTOK = tokens held in registers per pass.
    int cpt = 0, ntok = 1, nct = 0, cap = 0;
    for (int c = 1; c <= 4 && !cpt; c *= 2) {
        int nt = 1;
        if (c == 1) nt = tokens >= 3 ? 4 : tokens;
        else if (c == 2) nt = tokens >= 2 ? 2 : 1;
        const int cp = (c * nt >= 4) ? 256 : 384;
        const int n = (((units + c - 1) / c) + 31) / 32 * 32;
        if (n + 32 <= cp) { cpt = c; ntok = nt; nct = n; cap = cp; }
    }
    if (!cpt) return cudaErrorInvalidValue;
    // bytes between rows: packed, or a caller's padded stride (the padding is never read)
    const int rb = row_stride ? (int)row_stride : (cols / vals) * bytes;
    if (rb < (cols / vals) * bytes) return cudaErrorInvalidValue;
    int rpg = 1;
    if (cpt * ntok == 1) {
        if (g_rpg_max >= 4 && 4 * rb <= g_stage_target / 2) rpg = 4;
        else if (g_rpg_max >= 2 && 2 * rb <= g_stage_target / 2) rpg = 2;
    }
    int groups = std::max(1, std::min({(cap - 32) / nct, 15, g_stage_target / (rpg * rb)}));
    const int stage_rows = groups * rpg;
    const int stage_bytes = ((stage_rows * rb + 64) + 127) / 128 * 128;
    const int npass = (tokens + ntok - 1) / ntok;
    const int slot_bytes = npass * groups * (nct / 32) * rpg * ntok * 4;
    const size_t xbytes = (size_t)tokens * units * nx * 4 + 16;
    int stages = g_stages;
    auto smem_of = [&](int stg) { return 128 + (size_t)stg * slot_bytes + xbytes + 128 + (size_t)stg * stage_bytes; };
    while (stages > 2 && smem_of(stages) > 220 * 1024) --stages;
    const size_t smem = smem_of(stages);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;

    GemvArgs a = {};
    a.w = static_cast<const uint8_t *>(w);
    a.x = x;
    a.y = y;
    a.ys_t = ys_t;
    a.ys_r = ys_r;
    a.rows = rows;
    a.cols = cols;
    a.tokens = tokens;
    a.rb = rb;
    a.units = units;
    a.nct = nct;
    a.groups = groups;
    a.stage_rows = stage_rows;
    a.stage_bytes = stage_bytes;
    a.stages = stages;
    a.err = err;
    a.grp_off = grp_off;
    a.w_group_stride = w_group_stride;
    a.grp_rows = grp_rows;
    a.n_groups = n_groups;
    a.active_groups = std::max(1, std::min(active_groups, std::max(1, n_groups)));
    const int threads = groups * nct + 32;
    const bool al = (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (rb & 15) == 0 && (w_group_stride & 15) == 0;
    switch (type) {
    case T_Q4_K: return run_type<T_Q4_K>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    case T_Q5_K: return run_type<T_Q5_K>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    case T_Q6_K: return run_type<T_Q6_K>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    case T_Q8_0: return run_type<T_Q8_0>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    case T_Q4_0: return run_type<T_Q4_0>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    default: return cudaErrorInvalidValue;
    }
}

// Returns cudaErrorInvalidValue for unsupported shapes (cols not a multiple
// of the block size, or rows too wide for the register budget).  Token
// batches whose quantised activations do not fit in shared memory next to the
// weight pipeline are processed in chunks of tokens (one launch each).
bool gemv_mma_supported(int type, const void *w, int rows, int cols, int tokens);
cudaError_t launch_gemv_mma(const void *w, const float *x, float *y, long long ys_r, int rows, int cols, int *err,
                            int num_sms, cudaStream_t st);

// Unquantised weights (GGML F32 = 0, F16 = 1; engine/gguf_parser.py:180-288
// takes those through NumPy): y[t * ys_t + r * ys_r] = sum_c W[r, c] x[t, c],
// f32 accumulation.  One warp per row and up to 8 tokens per pass: the row
// streams once per pass with 16-byte loads (8 halves or 4 floats per lane per
// load), x rows come from L1/L2.  cols a multiple of 8.
template <typename TW>
__global__ void __launch_bounds__(256) gemv_dense_kernel(const TW *__restrict__ w, const float *__restrict__ x,
                                                         float *__restrict__ y, long long ys_t, long long ys_r,
                                                         int rows, int cols, int tokens)
{
    const long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const TW *wr = w + r * cols;
    for (int t0 = 0; t0 < tokens; t0 += 8) {
        const int nt = min(8, tokens - t0);
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int c = lane * 8; c < cols; c += 256) {
            float wv[8];
            if constexpr (sizeof(TW) == 2) {
                const uint4 u = __ldg(reinterpret_cast<const uint4 *>(wr + c));
                const uint32_t uw[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    wv[2 * i] = h2f(uw[i]);
                    wv[2 * i + 1] = h2f(uw[i] >> 16);
                }
            } else {
                const float4 a = __ldg(reinterpret_cast<const float4 *>(wr + c));
                const float4 b = __ldg(reinterpret_cast<const float4 *>(wr + c + 4));
                wv[0] = a.x; wv[1] = a.y; wv[2] = a.z; wv[3] = a.w;
                wv[4] = b.x; wv[5] = b.y; wv[6] = b.z; wv[7] = b.w;
            }
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                if (t >= nt) break;
                const float *xr = x + (long long)(t0 + t) * cols + c;
                const float4 a = __ldg(reinterpret_cast<const float4 *>(xr));
                const float4 b = __ldg(reinterpret_cast<const float4 *>(xr + 4));
                acc[t] = fmaf(wv[0], a.x, fmaf(wv[1], a.y, fmaf(wv[2], a.z, fmaf(wv[3], a.w, acc[t]))));
                acc[t] = fmaf(wv[4], b.x, fmaf(wv[5], b.y, fmaf(wv[6], b.z, fmaf(wv[7], b.w, acc[t]))));
            }
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            float v = acc[t];
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0 && t < nt) y[(t0 + t) * ys_t + r * ys_r] = v;
        }
    }
}

cudaError_t launch_gemv(int type, const void *w, const float *x, float *y, long long ys_t, long long ys_r, int rows,
                        int cols, int tokens, int *err, int num_sms, cudaStream_t st)
{
    if (type == 0 || type == 1) {
        if (rows < 1 || tokens < 1 || cols < 8 || cols % 8 || (reinterpret_cast<uintptr_t>(w) & 15) ||
            (reinterpret_cast<uintptr_t>(x) & 15))
            return cudaErrorInvalidValue;
        const unsigned grid = (unsigned)(((long long)rows * 32 + 255) / 256);
        if (type == 1)
            gemv_dense_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half *>(w), x, y, ys_t, ys_r, rows,
                                                            cols, tokens);
        else
            gemv_dense_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float *>(w), x, y, ys_t, ys_r, rows, cols,
                                                           tokens);
        return cudaGetLastError();
    }
    const int vals = type_vals(type), bytes = type_bytes(type);
    if (!bytes || rows < 1 || tokens < 1 || cols < vals || cols % vals) return cudaErrorInvalidValue;
    // batch-1 Q4_K: the integer-tensor-core kernel (gemv_mma.cu)
    if (g_use_mma && gemv_mma_supported(type, w, rows, cols, tokens) && !(reinterpret_cast<uintptr_t>(x) & 15))
        return launch_gemv_mma(w, x, y, ys_r, rows, cols, err, num_sms, st);
    const int units = (cols / vals) * ((vals == 256) ? 4 : 1);
    const size_t per_tok = (size_t)units * ((vals == 256) ? XPackWords<16>::N : XPackWords<8>::N) * 4;
    int chunk = (int)std::max<size_t>(1, (96 * 1024) / per_tok);
    if (chunk > 64) chunk = 64;
    for (int t0 = 0; t0 < tokens; t0 += chunk) {
        const int n = std::min(chunk, tokens - t0);
        cudaError_t e = launch_gemv_chunk(type, w, x + (long long)t0 * cols, y + t0 * ys_t, ys_t, ys_r, rows, cols, n,
                                          err, num_sms, st);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

// Grouped launch: for every group g with tokens (grp_off[g+1] - grp_off[g],
// at most max_tokens <= 64), y[grp_off[g] + t, r] = sum_c W_g[r, c] * x[grp_off[g] + t, c]
// with W_g at w + g * w_group_stride.  Groups without tokens read nothing.
int gemv_grouped_max_tokens(int type, int cols)
{
    const int vals = type_vals(type), bytes = type_bytes(type);
    if (!bytes || cols < vals || cols % vals) return 0;
    const int units = (cols / vals) * ((vals == 256) ? 4 : 1);
    const size_t per_tok = (size_t)units * ((vals == 256) ? XPackWords<16>::N : XPackWords<8>::N) * 4;
    return (int)std::min<size_t>(64, (128 * 1024) / per_tok);
}

cudaError_t launch_gemv_grouped(int type, const void *w, long long w_group_stride, int n_groups, const int *grp_off,
                                const float *x, float *y, long long ys_t, int rows, int cols, int max_tokens,
                                int x_rows, int active_groups, long long row_stride, int *err, int num_sms,
                                cudaStream_t st)
{
    if (rows < 1 || max_tokens < 1 || n_groups < 1 || !grp_off || x_rows < 1 ||
        max_tokens > gemv_grouped_max_tokens(type, cols))
        return cudaErrorInvalidValue;
    return launch_gemv_chunk(type, w, x, y, ys_t, 1, rows, cols, max_tokens, err, num_sms, st, grp_off,
                             w_group_stride, n_groups, active_groups, row_stride, x_rows);
}

} // namespace b200q
