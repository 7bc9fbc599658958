// Decode GEMV / small-batch matmul over raw GGML block-quant rows (sm_100a).
//
// y[t, r] = sum_c W[r, c] * x[t, c] for W stored as the raw GGUF bytes of a
// [rows, cols] Q4_0/Q8_0/Q4_K/Q5_K/Q6_K matrix -- the computation of
// localai_*_matvec / localai_*_matmul in the reference
// (engine/native_quant.cpp:126-337 row kernels, :705-768 exports), with the
// activation kept in f32 (the reference quantises it to int8/int16).
//
// Design (HBM-bound; ~0.56 B of weight per value for Q4_K):
// * One producer thread per CTA streams contiguous row tiles of the raw bytes
//   into a ring of shared-memory stages with non-tensor bulk copies
//   (cp.async.bulk, mbarrier complete_tx).  Any sub-16-byte tail is copied by
//   the producer with plain loads before it arrives on the stage barrier.
// * Consumer threads are "column stationary": a group of threads covers one
//   full row, each thread owning CPT fixed 32-value units of the row; the
//   x values of its units stay in registers for the whole kernel.  Groups
//   take different rows of a stage.  x is therefore read once per CTA and the
//   only shared-memory traffic is the weight stream itself.
// * A 4/5/6-bit quant q becomes the float 32768 + 256*q with one byte
//   permute (the byte lands in mantissa bits 16..23 under exponent 2^15), so
//   sum(q*x) = S/256 - 128*sum(x) with S accumulated by plain f32 FMAs.  The
//   per-unit sums of x are precomputed once.  Q8_0 uses the exact product
//   256*q*x.  Scales are applied once per 16-value run, in f32.
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
    int units;            // 32-value units per row
    int nct;              // consumer threads per group (multiple of 32)
    int groups;           // row groups per CTA
    int stage_rows;       // groups * RPG
    int stage_bytes;      // bytes per shared stage buffer
    int stages;
    int *err;
};

constexpr uint32_t MAGIC_B2 = 0x47000000u;   // exponent 2^15; byte 2 = q -> 32768 + 256 q

__device__ __forceinline__ float qf(uint32_t bytes4, int b)
{
    return __uint_as_float(__byte_perm(bytes4, MAGIC_B2, 0x7044u | (uint32_t)(b << 8)));
}

// Column start of the low and high 16-value runs of unit u.
template <int T>
__device__ __forceinline__ void unit_cols(int u, int &lo, int &hi)
{
    if constexpr (T == T_Q4_K || T == T_Q5_K) {
        const int blk = u >> 3, c = u & 7;
        lo = blk * 256 + 64 * (c >> 1) + 16 * (c & 1);
        hi = lo + 32;
    } else if constexpr (T == T_Q6_K) {
        const int blk = u >> 3, c = u & 7;
        lo = blk * 256 + 128 * (c >> 2) + 32 * ((c >> 1) & 1) + 16 * (c & 1);
        hi = lo + 64;
    } else {
        lo = u * 32;
        hi = lo + 16;
    }
}

// 32 bytes from any shared address (9 aligned words + funnel shifts).
__device__ __forceinline__ void lds256_any(uint32_t a, uint32_t o[8])
{
    const uint32_t base = a & ~3u, sh = (a & 3u) * 8u;
    uint32_t w[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) w[i] = lds32(base + 4 * i);
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = __funnelshift_r(w[i], w[i + 1], sh);
}

// ---------------------------------------------------------------- unit dots
// Each adds the unit's contribution for NTOK tokens into acc[].
// blk: shared address of the block start; c: unit index inside the block.

template <int NTOK, bool AL>
__device__ __forceinline__ void dot_q4k(uint32_t blk, int c, const float (&x)[NTOK][32],
                                        const float (&xs)[NTOK][2], float (&acc)[NTOK])
{
    const uint4 hdr = lds128_any<AL>(blk);
    const uint4 q = lds128_any<AL>(blk + 16 + 16 * c);
    const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
    // 6-bit scale/min of sub-blocks k0 = 2*(c>>1) and k0+1 (engine/dequant.py:108-113)
    const bool hk = c >= 4;
    const int k0 = 2 * (c >> 1);
    const int o0 = 8 * (k0 & 3), o1 = o0 + 8;
    const uint32_t as = hk ? hdr.w : hdr.y, am = hk ? hdr.w : hdr.z;
    const int mo = hk ? 4 : 0, ho = hk ? 6 : 4;
    const uint32_t sc0 = ((as >> o0) & 15u) | (((hdr.y >> (o0 + ho)) & 3u) << 4);
    const uint32_t sc1 = ((as >> o1) & 15u) | (((hdr.y >> (o1 + ho)) & 3u) << 4);
    const uint32_t mn0 = ((am >> (o0 + mo)) & 15u) | (((hdr.z >> (o0 + ho)) & 3u) << 4);
    const uint32_t mn1 = ((am >> (o1 + mo)) & 15u) | (((hdr.z >> (o1 + ho)) & 3u) << 4);
    const float ds0 = d * (float)sc0, ds1 = d * (float)sc1;
    const float dm0 = dmin * (float)mn0, dm1 = dmin * (float)mn1;
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    float s0[NTOK], s1[NTOK];
#pragma unroll
    for (int t = 0; t < NTOK; ++t) s0[t] = s1[t] = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t lo = qw[w] & 0x0F0F0F0Fu, hi = (qw[w] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const float flo = qf(lo, b), fhi = qf(hi, b);
#pragma unroll
            for (int t = 0; t < NTOK; ++t) {
                s0[t] = fmaf(flo, x[t][4 * w + b], s0[t]);
                s1[t] = fmaf(fhi, x[t][16 + 4 * w + b], s1[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
        const float a0 = fmaf(s0[t], 1.0f / 256.0f, -128.0f * xs[t][0]);   // sum q*x, low run
        const float a1 = fmaf(s1[t], 1.0f / 256.0f, -128.0f * xs[t][1]);
        acc[t] += (ds0 * a0 + ds1 * a1) - (dm0 * xs[t][0] + dm1 * xs[t][1]);
    }
}

template <int NTOK, bool AL>
__device__ __forceinline__ void dot_q5k(uint32_t blk, int c, const float (&x)[NTOK][32],
                                        const float (&xs)[NTOK][2], float (&acc)[NTOK])
{
    const uint4 hdr = lds128_any<AL>(blk);
    const uint4 qh = lds128_any<AL>(blk + 16 + 16 * (c & 1));
    const uint4 q = lds128_any<AL>(blk + 48 + 16 * c);
    const float d = h2f(hdr.x), dmin = h2f(hdr.x >> 16);
    const bool hk = c >= 4;
    const int k0 = 2 * (c >> 1);
    const int o0 = 8 * (k0 & 3), o1 = o0 + 8;
    const uint32_t as = hk ? hdr.w : hdr.y, am = hk ? hdr.w : hdr.z;
    const int mo = hk ? 4 : 0, ho = hk ? 6 : 4;
    const uint32_t sc0 = ((as >> o0) & 15u) | (((hdr.y >> (o0 + ho)) & 3u) << 4);
    const uint32_t sc1 = ((as >> o1) & 15u) | (((hdr.y >> (o1 + ho)) & 3u) << 4);
    const uint32_t mn0 = ((am >> (o0 + mo)) & 15u) | (((hdr.z >> (o0 + ho)) & 3u) << 4);
    const uint32_t mn1 = ((am >> (o1 + mo)) & 15u) | (((hdr.z >> (o1 + ho)) & 3u) << 4);
    const float ds0 = d * (float)sc0, ds1 = d * (float)sc1;
    const float dm0 = dmin * (float)mn0, dm1 = dmin * (float)mn1;
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
    float s0[NTOK], s1[NTOK];
#pragma unroll
    for (int t = 0; t < NTOK; ++t) s0[t] = s1[t] = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t lo = (qw[w] & 0x0F0F0F0Fu) | (((hw[w] >> k0) & 0x01010101u) << 4);
        const uint32_t hi = ((qw[w] >> 4) & 0x0F0F0F0Fu) | (((hw[w] >> (k0 + 1)) & 0x01010101u) << 4);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const float flo = qf(lo, b), fhi = qf(hi, b);
#pragma unroll
            for (int t = 0; t < NTOK; ++t) {
                s0[t] = fmaf(flo, x[t][4 * w + b], s0[t]);
                s1[t] = fmaf(fhi, x[t][16 + 4 * w + b], s1[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
        const float a0 = fmaf(s0[t], 1.0f / 256.0f, -128.0f * xs[t][0]);
        const float a1 = fmaf(s1[t], 1.0f / 256.0f, -128.0f * xs[t][1]);
        acc[t] += (ds0 * a0 + ds1 * a1) - (dm0 * xs[t][0] + dm1 * xs[t][1]);
    }
}

template <int NTOK>
__device__ __forceinline__ void dot_q6k(uint32_t blk, int c, const float (&x)[NTOK][32],
                                        const float (&xs)[NTOK][2], float (&acc)[NTOK])
{
    const int h = c >> 2, a = (c >> 1) & 1, jh = c & 1;
    const uint4 ql = lds128_any<false>(blk + 64 * h + 32 * a + 16 * jh);
    const uint4 qh = lds128_any<false>(blk + 128 + 32 * h + 16 * jh);
    const uint32_t sb = blk + 192 + 8 * h + 2 * a + jh;
    const float sc0 = (float)(int8_t)lds_u8(sb), sc1 = (float)(int8_t)lds_u8(sb + 4);
    const float d = h2f(lds_u16(blk + 208));
    const int shl = 4 - 2 * a, shr = 2 * a;
    const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w};
    const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
    float s0[NTOK], s1[NTOK];
#pragma unroll
    for (int t = 0; t < NTOK; ++t) s0[t] = s1[t] = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t lo = (lw[w] & 0x0F0F0F0Fu) | ((hw[w] << shl) & 0x30303030u);
        const uint32_t hi = ((lw[w] >> 4) & 0x0F0F0F0Fu) | ((hw[w] >> shr) & 0x30303030u);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const float flo = qf(lo, b), fhi = qf(hi, b);
#pragma unroll
            for (int t = 0; t < NTOK; ++t) {
                s0[t] = fmaf(flo, x[t][4 * w + b], s0[t]);
                s1[t] = fmaf(fhi, x[t][16 + 4 * w + b], s1[t]);
            }
        }
    }
    const float ds0 = d * sc0, ds1 = d * sc1;
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
        // sum (q-32)*x = S/256 - 128*X - 32*X
        const float a0 = fmaf(s0[t], 1.0f / 256.0f, -160.0f * xs[t][0]);
        const float a1 = fmaf(s1[t], 1.0f / 256.0f, -160.0f * xs[t][1]);
        acc[t] += ds0 * a0 + ds1 * a1;
    }
}

template <int NTOK>
__device__ __forceinline__ void dot_q8_0(uint32_t blk, const float (&x)[NTOK][32], float (&acc)[NTOK])
{
    const float d = h2f(lds_u16(blk));
    uint32_t qw[8];
    lds256_any(blk + 2, qw);
    float s[NTOK];
#pragma unroll
    for (int t = 0; t < NTOK; ++t) s[t] = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const uint32_t v = qw[w] ^ 0x80808080u;     // q + 128 as unsigned bytes
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            // 2^23 + 256*(q+128), minus 2^23 + 32768 -> exactly 256*q
            const float f = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7404u | (uint32_t)(b << 4))) - 8421376.0f;
#pragma unroll
            for (int t = 0; t < NTOK; ++t) s[t] = fmaf(f, x[t][4 * w + b], s[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < NTOK; ++t) acc[t] = fmaf(d * (1.0f / 256.0f), s[t], acc[t]);
}

template <int NTOK>
__device__ __forceinline__ void dot_q4_0(uint32_t blk, const float (&x)[NTOK][32], const float (&xs)[NTOK][2],
                                         float (&acc)[NTOK])
{
    const float d = h2f(lds_u16(blk));
    const uint4 q = lds128_any<false>(blk + 2);
    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
    float s0[NTOK], s1[NTOK];
#pragma unroll
    for (int t = 0; t < NTOK; ++t) s0[t] = s1[t] = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        const uint32_t lo = qw[w] & 0x0F0F0F0Fu, hi = (qw[w] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const float flo = qf(lo, b), fhi = qf(hi, b);
#pragma unroll
            for (int t = 0; t < NTOK; ++t) {
                s0[t] = fmaf(flo, x[t][4 * w + b], s0[t]);
                s1[t] = fmaf(fhi, x[t][16 + 4 * w + b], s1[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < NTOK; ++t) {
        // sum (q-8)*x = S/256 - 128*X - 8*X
        const float a0 = fmaf(s0[t], 1.0f / 256.0f, -136.0f * xs[t][0]);
        const float a1 = fmaf(s1[t], 1.0f / 256.0f, -136.0f * xs[t][1]);
        acc[t] = fmaf(d, a0 + a1, acc[t]);
    }
}

template <int T, int NTOK, bool AL>
__device__ __forceinline__ void unit_dot(uint32_t blk, int c, const float (&x)[NTOK][32], const float (&xs)[NTOK][2],
                                         float (&acc)[NTOK])
{
    if constexpr (T == T_Q4_K) dot_q4k<NTOK, AL>(blk, c, x, xs, acc);
    else if constexpr (T == T_Q5_K) dot_q5k<NTOK, AL>(blk, c, x, xs, acc);
    else if constexpr (T == T_Q6_K) dot_q6k<NTOK>(blk, c, x, xs, acc);
    else if constexpr (T == T_Q8_0) dot_q8_0<NTOK>(blk, x, acc);
    else dot_q4_0<NTOK>(blk, x, xs, acc);
}

// ---------------------------------------------------------------- kernel
// Shared layout: [full mbarriers][empty mbarriers] (128 B) | reduction
// buffers | stage buffers (128-B aligned).
// Thread cap per configuration so that the stationary x registers
// (32 * CPT * NTOK floats) fit without spilling.
template <int CPT, int NTOK>
struct GemvCap { static constexpr int THREADS = (CPT * NTOK >= 4) ? 256 : (CPT * NTOK == 2 ? 384 : 544); };

template <int T, int CPT, int NTOK, int RPG, bool AL>
__global__ void __launch_bounds__(GemvCap<CPT, NTOK>::THREADS) gemv_kernel(const GemvArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int UPB = Fmt<T>::UPB, BYTES = Fmt<T>::BYTES;
    const int tid = threadIdx.x;
    const int ncons = a.groups * a.nct;
    const uint32_t sbase = smem_addr(smem);
    const uint32_t full0 = sbase, empty0 = sbase + 8 * a.stages;
    float *red = reinterpret_cast<float *>(smem + 128);
    const int nwg = a.nct >> 5;                                  // warps per group
    const int red_per_buf = a.groups * nwg * RPG * NTOK;
    const uint32_t stage0 = (sbase + 128 + 2 * red_per_buf * 4 + 127) & ~127u;

    const long long r_begin = (long long)blockIdx.x * a.rows / gridDim.x;
    const long long r_end = (long long)(blockIdx.x + 1) * a.rows / gridDim.x;
    const int n_it = (int)((r_end - r_begin + a.stage_rows - 1) / a.stage_rows);

    if (tid == 0) {
        for (int s = 0; s < a.stages; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, ncons / 32);
        }
        mbar_fence_init();
    }
    __syncthreads();

    if (tid >= ncons) {                        // ---- producer warp
        if (tid != ncons) return;
        const uint64_t pol = policy_evict_first();
        int it = 0;
        bool ok = true;
        for (; it < n_it && ok; ++it) {
            const int s = it % a.stages;
            if (it >= a.stages && !mbar_wait(empty0 + 8 * s, ((it / a.stages) + 1) & 1, a.err)) {
                ok = false;
                break;
            }
            const long long row0 = r_begin + (long long)it * a.stage_rows;
            const int nr = (int)min((long long)a.stage_rows, r_end - row0);
            const uint8_t *gs = a.w + row0 * a.rb;
            const uint8_t *ge = gs + (long long)nr * a.rb;
            const uint8_t *a0 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(gs) & ~(uintptr_t)15);
            const uint8_t *a1 = reinterpret_cast<const uint8_t *>(reinterpret_cast<uintptr_t>(ge) & ~(uintptr_t)15);
            const uint32_t dst = stage0 + (uint32_t)s * a.stage_bytes;
            for (const uint8_t *p = a1; p < ge; ++p)              // < 16 tail bytes
                asm volatile("st.shared.u8 [%0], %1;" ::"r"(dst + (uint32_t)(p - a0)), "h"((unsigned short)__ldg(p)));
            const uint32_t nbytes = (uint32_t)(a1 - a0);
            if (nbytes) {
                mbar_arrive_expect_tx(full0 + 8 * s, nbytes);
                bulk_g2s(dst, a0, nbytes, full0 + 8 * s, pol);
            } else {
                mbar_arrive(full0 + 8 * s);
            }
        }
        if (!ok) {                                // drain copies already issued
            for (int j = max(0, it - a.stages); j < it; ++j)
                mbar_wait(full0 + 8 * (j % a.stages), (j / a.stages) & 1, a.err);
        }
        return;
    }

    // ---- consumers
    const int g = tid / a.nct, lt = tid % a.nct;
    const int wig = lt >> 5, lane = tid & 31;
    int ucol_lo[CPT], ucol_hi[CPT], uoff[CPT], uc[CPT];
    bool uval[CPT];
#pragma unroll
    for (int i = 0; i < CPT; ++i) {
        const int u = lt + i * a.nct;
        uval[i] = u < a.units;
        const int uu = uval[i] ? u : 0;
        unit_cols<T>(uu, ucol_lo[i], ucol_hi[i]);
        uoff[i] = (uu / UPB) * BYTES;
        uc[i] = uu % UPB;
    }
    float x[CPT][NTOK][32];
    float xs[CPT][NTOK][2];
    const int npass = (a.tokens + NTOK - 1) / NTOK;

    auto load_x = [&](int pass) {
#pragma unroll
        for (int i = 0; i < CPT; ++i)
#pragma unroll
            for (int t = 0; t < NTOK; ++t) {
                const int tok = pass * NTOK + t;
                const bool v = uval[i] && tok < a.tokens;
                const float *xl = a.x + (long long)(v ? tok : 0) * a.cols;
                float slo = 0.f, shi = 0.f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    float4 l = v ? __ldg(reinterpret_cast<const float4 *>(xl + ucol_lo[i]) + q) : make_float4(0, 0, 0, 0);
                    float4 h = v ? __ldg(reinterpret_cast<const float4 *>(xl + ucol_hi[i]) + q) : make_float4(0, 0, 0, 0);
                    x[i][t][4 * q + 0] = l.x; x[i][t][4 * q + 1] = l.y; x[i][t][4 * q + 2] = l.z; x[i][t][4 * q + 3] = l.w;
                    x[i][t][16 + 4 * q + 0] = h.x; x[i][t][16 + 4 * q + 1] = h.y;
                    x[i][t][16 + 4 * q + 2] = h.z; x[i][t][16 + 4 * q + 3] = h.w;
                    slo += (l.x + l.y) + (l.z + l.w);
                    shi += (h.x + h.y) + (h.z + h.w);
                }
                xs[i][t][0] = slo;
                xs[i][t][1] = shi;
            }
    };
    if (npass == 1) load_x(0);

    int rbuf = 0;
    for (int it = 0; it < n_it; ++it) {
        const int s = it % a.stages;
        if (!mbar_wait(full0 + 8 * s, (it / a.stages) & 1, a.err)) return;
        const long long row0 = r_begin + (long long)it * a.stage_rows;
        const int nr = (int)min((long long)a.stage_rows, r_end - row0);
        const uintptr_t gs = reinterpret_cast<uintptr_t>(a.w + row0 * a.rb);
        const uint32_t base = stage0 + (uint32_t)s * a.stage_bytes + (uint32_t)(gs & 15);

        for (int pass = 0; pass < npass; ++pass) {
            if (npass > 1) load_x(pass);
            float acc[RPG][NTOK];
#pragma unroll
            for (int rr = 0; rr < RPG; ++rr)
#pragma unroll
                for (int t = 0; t < NTOK; ++t) acc[rr][t] = 0.f;
#pragma unroll
            for (int rr = 0; rr < RPG; ++rr) {
                const int lr = g + rr * a.groups;
                if (lr < nr) {
                    const uint32_t rbase = base + (uint32_t)(lr * a.rb);
#pragma unroll
                    for (int i = 0; i < CPT; ++i)
                        if (uval[i]) unit_dot<T, NTOK, AL>(rbase + uoff[i], uc[i], x[i], xs[i], acc[rr]);
                }
            }
            if (pass == npass - 1) {              // stage fully read by this warp
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * s);
            }
            // warp reduction
#pragma unroll
            for (int rr = 0; rr < RPG; ++rr)
#pragma unroll
                for (int t = 0; t < NTOK; ++t) {
                    float v = acc[rr][t];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    acc[rr][t] = v;
                }
            if (nwg == 1) {
                if (lane == 0) {
#pragma unroll
                    for (int rr = 0; rr < RPG; ++rr) {
                        const int lr = g + rr * a.groups;
#pragma unroll
                        for (int t = 0; t < NTOK; ++t) {
                            const int tok = pass * NTOK + t;
                            if (lr < nr && tok < a.tokens) a.y[tok * a.ys_t + (row0 + lr) * a.ys_r] = acc[rr][t];
                        }
                    }
                }
            } else {
                float *rb = red + rbuf * red_per_buf + ((g * nwg + wig) * RPG) * NTOK;
                if (lane == 0) {
#pragma unroll
                    for (int rr = 0; rr < RPG; ++rr)
#pragma unroll
                        for (int t = 0; t < NTOK; ++t) rb[rr * NTOK + t] = acc[rr][t];
                }
                named_bar_sync(1 + g, a.nct);
                if (lt < RPG * NTOK) {
                    const int rr = lt / NTOK, t = lt % NTOK;
                    const int lr = g + rr * a.groups;
                    const int tok = pass * NTOK + t;
                    const float *gb = red + rbuf * red_per_buf + (g * nwg) * RPG * NTOK;
                    float v = 0.f;
                    for (int wv = 0; wv < nwg; ++wv) v += gb[wv * RPG * NTOK + lt];
                    if (lr < nr && tok < a.tokens) a.y[tok * a.ys_t + (row0 + lr) * a.ys_r] = v;
                }
                rbuf ^= 1;
            }
        }
    }
}

// ---------------------------------------------------------------- host side
struct GemvPlan {
    int cpt, ntok, rpg;
    GemvArgs a;
    size_t smem;
    int threads;
};

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
    const int per_sm = occ_per_sm;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const long long tiles = (a.rows + a.stage_rows - 1) / a.stage_rows;
    long long grid = (long long)num_sms * per_sm;
    if (grid > tiles) grid = tiles;
    kern<<<(int)grid, threads, smem, st>>>(a);
    return cudaGetLastError();
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
    switch (rpg) {
    case 1: return run_al<T, CPT, NTOK, 1>(a, threads, smem, num_sms, st, al);
    case 2: return run_al<T, CPT, NTOK, 2>(a, threads, smem, num_sms, st, al);
    default: return run_al<T, CPT, NTOK, 4>(a, threads, smem, num_sms, st, al);
    }
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

// Tuning knobs (defaults chosen on B200): target bytes of weights per stage
// and number of stages.
static int g_stage_target = 24 * 1024;
static int g_stages = 4;
void gemv_set_tuning(int stage_target_bytes, int stages)
{
    if (stage_target_bytes > 0) g_stage_target = stage_target_bytes;
    if (stages > 0) g_stages = stages;
}

// Returns cudaErrorInvalidValue for unsupported shapes (cols not a multiple
// of the block size, or more than 65536 columns).
cudaError_t launch_gemv(int type, const void *w, const float *x, float *y, long long ys_t, long long ys_r, int rows,
                        int cols, int tokens, int *err, int num_sms, cudaStream_t st)
{
    const int vals = type_vals(type), bytes = type_bytes(type);
    if (!bytes || rows < 1 || tokens < 1 || cols < vals || cols % vals) return cudaErrorInvalidValue;
    const int upb = (vals == 256) ? 8 : 1;
    const int units = (cols / vals) * upb;
    // Smallest units-per-thread (CPT) whose group fits the thread cap of its
    // register budget; NTOK = tokens held in registers per pass.
    int cpt = 0, ntok = 1, nct = 0, cap = 0;
    for (int c = 1; c <= 4 && !cpt; c *= 2) {
        int nt = 1;
        if (c == 1) nt = tokens >= 3 ? 4 : tokens;
        else if (c == 2) nt = tokens >= 2 ? 2 : 1;
        const int cp = (c * nt >= 4) ? 256 : (c * nt == 2 ? 384 : 544);
        const int n = (((units + c - 1) / c) + 31) / 32 * 32;
        if (n + 32 <= cp) { cpt = c; ntok = nt; nct = n; cap = cp; }
    }
    if (!cpt) return cudaErrorInvalidValue;
    const int rb = (cols / vals) * bytes;
    int rpg = 1;
    if (4 * rb <= g_stage_target / 2) rpg = 4;
    else if (2 * rb <= g_stage_target / 2) rpg = 2;
    int groups = std::max(1, std::min({(cap - 32) / nct, 15, g_stage_target / (rpg * rb)}));
    const int stage_rows = groups * rpg;
    const int stage_bytes = ((stage_rows * rb + 64) + 127) / 128 * 128;
    const int nwg = nct / 32;
    const int red_bytes = 2 * groups * nwg * rpg * ntok * 4;
    int stages = g_stages;
    const size_t fixed = 128 + red_bytes + 128;
    while (stages > 2 && fixed + (size_t)stages * stage_bytes > 220 * 1024) --stages;
    const size_t smem = fixed + (size_t)stages * stage_bytes;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;

    GemvArgs a;
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
    const int threads = groups * nct + 32;
    const bool al = (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (rb & 15) == 0;
    switch (type) {
    case T_Q4_K: return run_type<T_Q4_K>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    case T_Q5_K: return run_type<T_Q5_K>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    case T_Q6_K: return run_type<T_Q6_K>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    case T_Q8_0: return run_type<T_Q8_0>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    case T_Q4_0: return run_type<T_Q4_0>(a, cpt, ntok, rpg, threads, smem, num_sms, st, al);
    default: return cudaErrorInvalidValue;
    }
}

} // namespace b200q
