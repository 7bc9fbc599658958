// Bit-exact GGML block dequantization on the GPU.
//
// Reproduces engine/dequant.py:dequantize of the reference (Q4_0 :62-66,
// Q8_0 :75-78, Q4_K :97-120, Q5_K :122-144, Q6_K :146-167) value for value:
// each product of the reference formula is exact in f32, and the Q4_K/Q5_K
// minimum term is subtracted with one round-to-nearest, so the explicit
// __fmul_rn/__fsub_rn below give the same f32 bits (FMA contraction, which
// would not change these exact products either, is ruled out explicitly).
//
// Work split: one thread decodes one run of 32 consecutive output values
// (one Q4_K/Q5_K/Q6_K sub-block or one Q8_0/Q4_0 block) and writes it with
// four 16-byte stores per 16 values.  The kernel is HBM-bound: it reads
// BYTES/VALS bytes and writes 4 bytes (f32) or 2 bytes (bf16) per value.
#include "common.cuh"

namespace b200q {

__device__ __forceinline__ uint32_t ldb(const uint8_t *p) { return __ldg(p); }
__device__ __forceinline__ float ldh(const uint8_t *p) { return h2f(ldb(p) | (ldb(p + 1) << 8)); }

__device__ __forceinline__ void k_scale_min(const uint8_t *s, int g, uint32_t &sc, uint32_t &mn)
{
    if (g < 4) {
        sc = ldb(s + g) & 63u;
        mn = ldb(s + g + 4) & 63u;
    } else {
        sc = (ldb(s + g + 4) & 15u) | ((ldb(s + g - 4) >> 6) << 4);
        mn = (ldb(s + g + 4) >> 4) | ((ldb(s + g) >> 6) << 4);
    }
}

// Decode values [32*r, 32*r+32) of one block into v[].
template <int T>
__device__ __forceinline__ void decode_run(const uint8_t *blk, int r, float v[32])
{
    if constexpr (T == T_Q8_0) {
        const float d = ldh(blk);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = __fmul_rn((float)(int8_t)ldb(blk + 2 + i), d);
    } else if constexpr (T == T_Q4_0) {
        const float d = ldh(blk);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const uint32_t b = ldb(blk + 2 + i);
            v[i] = __fmul_rn(__fsub_rn((float)(b & 15u), 8.0f), d);
            v[i + 16] = __fmul_rn(__fsub_rn((float)(b >> 4), 8.0f), d);
        }
    } else if constexpr (T == T_Q4_K || T == T_Q5_K) {
        const float d = ldh(blk), dmin = ldh(blk + 2);
        uint32_t sc, mn;
        k_scale_min(blk + 4, r, sc, mn);
        const float step = __fmul_rn(d, (float)sc);
        const float low = __fmul_rn(dmin, (float)mn);
        const uint8_t *qs = blk + (T == T_Q4_K ? 16 : 48) + (r / 2) * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            uint32_t q = ldb(qs + j);
            q = (r & 1) ? (q >> 4) : (q & 15u);
            if constexpr (T == T_Q5_K) q |= ((ldb(blk + 16 + j) >> r) & 1u) << 4;
            v[j] = __fsub_rn(__fmul_rn((float)q, step), low);
        }
    } else {  // Q6_K: r = 4*half + quad
        const int h = r >> 2, u = r & 3;
        const float d = ldh(blk + 208);
        const uint8_t *ql = blk + 64 * h + 32 * (u & 1);
        const uint8_t *qh = blk + 128 + 32 * h;
        const float s0 = (float)(int8_t)ldb(blk + 192 + 8 * h + 2 * u);
        const float s1 = (float)(int8_t)ldb(blk + 192 + 8 * h + 2 * u + 1);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            uint32_t lo = ldb(ql + j);
            lo = (u < 2) ? (lo & 15u) : (lo >> 4);
            const uint32_t hi = (ldb(qh + j) >> (2 * u)) & 3u;
            const float q = (float)((int)(lo | (hi << 4)) - 32);
            v[j] = __fmul_rn(__fmul_rn(q, d), j < 16 ? s0 : s1);
        }
    }
}

template <int T, typename OutT>
__global__ void dequant_kernel(const uint8_t *__restrict__ raw, OutT *__restrict__ out, long long nruns)
{
    constexpr int RUNS = Fmt<T>::VALS / 32;
    for (long long run = blockIdx.x * (long long)blockDim.x + threadIdx.x; run < nruns;
         run += (long long)gridDim.x * blockDim.x) {
        const long long blk = run / RUNS;
        const int r = (int)(run % RUNS);
        float v[32];
        decode_run<T>(raw + blk * Fmt<T>::BYTES, r, v);
        OutT *o = out + run * 32;
        if constexpr (sizeof(OutT) == 4) {
            float4 *o4 = reinterpret_cast<float4 *>(o);
#pragma unroll
            for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
            uint4 *o4 = reinterpret_cast<uint4 *>(o);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint4 w;
                __nv_bfloat162 p0 = __floats2bfloat162_rn(v[8 * i], v[8 * i + 1]);
                __nv_bfloat162 p1 = __floats2bfloat162_rn(v[8 * i + 2], v[8 * i + 3]);
                __nv_bfloat162 p2 = __floats2bfloat162_rn(v[8 * i + 4], v[8 * i + 5]);
                __nv_bfloat162 p3 = __floats2bfloat162_rn(v[8 * i + 6], v[8 * i + 7]);
                w.x = *reinterpret_cast<uint32_t *>(&p0);
                w.y = *reinterpret_cast<uint32_t *>(&p1);
                w.z = *reinterpret_cast<uint32_t *>(&p2);
                w.w = *reinterpret_cast<uint32_t *>(&p3);
                o4[i] = w;
            }
        }
    }
}

template <typename OutT>
cudaError_t launch_dequant_t(int type, const void *raw, OutT *out, long long nblocks, int num_sms, cudaStream_t st)
{
    const long long runs = nblocks * (type_vals(type) / 32);
    if (runs <= 0) return cudaSuccess;
    const int threads = 256;
    long long grid = (runs + threads - 1) / threads;
    const long long cap = (long long)num_sms * 16;
    if (grid > cap) grid = cap;
    const uint8_t *r = static_cast<const uint8_t *>(raw);
    switch (type) {
    case T_Q4_0: dequant_kernel<T_Q4_0, OutT><<<(int)grid, threads, 0, st>>>(r, out, runs); break;
    case T_Q8_0: dequant_kernel<T_Q8_0, OutT><<<(int)grid, threads, 0, st>>>(r, out, runs); break;
    case T_Q4_K: dequant_kernel<T_Q4_K, OutT><<<(int)grid, threads, 0, st>>>(r, out, runs); break;
    case T_Q5_K: dequant_kernel<T_Q5_K, OutT><<<(int)grid, threads, 0, st>>>(r, out, runs); break;
    case T_Q6_K: dequant_kernel<T_Q6_K, OutT><<<(int)grid, threads, 0, st>>>(r, out, runs); break;
    default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t launch_dequant_f32(int type, const void *raw, float *out, long long nblocks, int num_sms, cudaStream_t st)
{
    return launch_dequant_t<float>(type, raw, out, nblocks, num_sms, st);
}
cudaError_t launch_dequant_bf16(int type, const void *raw, __nv_bfloat16 *out, long long nblocks, int num_sms,
                                cudaStream_t st)
{
    return launch_dequant_t<__nv_bfloat16>(type, raw, out, nblocks, num_sms, st);
}

// One row of a quantised [rows, cols] matrix, the row index read from device
// memory (the token embedding lookup of a decode step whose token is chosen on
// the device): out[c] = dequant(raw row *row_idx)[c], bit-exact as above.
template <int T>
__global__ void dequant_row_kernel(const uint8_t *__restrict__ raw, long long row_bytes, int cols,
                                   const int *__restrict__ row_idx, int rows, float *__restrict__ out, int *err)
{
    // blockIdx.y: which of the requested rows (row_idx[y] -> out row y)
    pdl_enter();
    const int r = row_idx[blockIdx.y];
    out += (long long)blockIdx.y * cols;
    if (r < 0 || r >= rows) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, ERR_BAD_INDEX);
        return;
    }
    const long long runs = cols / 32;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < runs; i += (long long)gridDim.x * blockDim.x) {
        const long long vals = Fmt<T>::VALS;
        const long long blk = (i * 32) / vals;
        const int sub = (int)((i * 32 - blk * vals) / 32);
        float v[32];
        decode_run<T>(raw + r * row_bytes + blk * Fmt<T>::BYTES, sub, v);
        float4 *o = reinterpret_cast<float4 *>(out + i * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) o[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
}

// The same lookup for unquantised rows (GGML F32 = 0, F16 = 1): a copy to f32.
template <typename TW>
__global__ void dense_row_kernel(const uint8_t *__restrict__ raw, long long row_bytes, int cols,
                                 const int *__restrict__ row_idx, int rows, float *__restrict__ out, int *err)
{
    pdl_enter();
    const int r = row_idx[blockIdx.y];
    out += (long long)blockIdx.y * cols;
    if (r < 0 || r >= rows) {
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, ERR_BAD_INDEX);
        return;
    }
    const TW *src = reinterpret_cast<const TW *>(raw + r * row_bytes);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < cols; i += (long long)gridDim.x * blockDim.x) {
        if constexpr (sizeof(TW) == 2) out[i] = __half2float(src[i]);
        else out[i] = src[i];
    }
}

cudaError_t launch_dequant_row(int type, const void *raw, long long row_bytes, int cols, const int *row_idx, int rows,
                               int n, float *out, int *err, cudaStream_t st)
{
    if (type == 0 || type == 1) {
        if (cols < 1 || n < 1 || n > 65535 || row_bytes < (long long)cols * (type == 0 ? 4 : 2)) return cudaErrorInvalidValue;
        const dim3 grid((cols + 255) / 256, n);
        const uint8_t *r = static_cast<const uint8_t *>(raw);
        if (type == 1)
            return launch_pdl(dense_row_kernel<__half>, grid, dim3(256), 0, st, r, row_bytes, cols, row_idx, rows, out,
                              err);
        return launch_pdl(dense_row_kernel<float>, grid, dim3(256), 0, st, r, row_bytes, cols, row_idx, rows, out, err);
    }
    if (cols < 32 || cols % type_vals(type) || n < 1 || n > 65535 || (reinterpret_cast<uintptr_t>(out) & 15))
        return cudaErrorInvalidValue;
    const int runs = cols / 32, threads = 128;
    const dim3 grid((runs + threads - 1) / threads, n);
    const uint8_t *r = static_cast<const uint8_t *>(raw);
    switch (type) {
    case T_Q4_0: return launch_pdl(dequant_row_kernel<T_Q4_0>, grid, dim3(threads), 0, st, r, row_bytes, cols, row_idx, rows, out, err);
    case T_Q8_0: return launch_pdl(dequant_row_kernel<T_Q8_0>, grid, dim3(threads), 0, st, r, row_bytes, cols, row_idx, rows, out, err);
    case T_Q4_K: return launch_pdl(dequant_row_kernel<T_Q4_K>, grid, dim3(threads), 0, st, r, row_bytes, cols, row_idx, rows, out, err);
    case T_Q5_K: return launch_pdl(dequant_row_kernel<T_Q5_K>, grid, dim3(threads), 0, st, r, row_bytes, cols, row_idx, rows, out, err);
    case T_Q6_K: return launch_pdl(dequant_row_kernel<T_Q6_K>, grid, dim3(threads), 0, st, r, row_bytes, cols, row_idx, rows, out, err);
    default: return cudaErrorInvalidValue;
    }
}

} // namespace b200q
