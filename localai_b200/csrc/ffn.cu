// Dense FFN glue for the decode path (engine/model.py:161-166, :230-233):
//   act[t, f] = silu(gate[t, f]) * up[t, f],  silu(g) = g / (1 + exp(-clip(g, -80, 80)))
// (act rows ld_out apart, so a zero-padded K tail can follow the F values)
// with gate and up read from one [T, 2F] f32 matrix (the output of a single
// GEMV over the concatenated [gate; up] weights).  HBM-bound elementwise.
#include "common.cuh"

namespace b200q {

__global__ void silu_mul_kernel(const float *__restrict__ gu, int T, int F, float *__restrict__ out, long long ld_out)
{
    pdl_enter();
    const long long n = (long long)T * F;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / F;
        const int f = (int)(i - t * F);
        out[t * ld_out + f] = silu_mul(gu[t * 2 * F + f], gu[t * 2 * F + F + f]);
    }
}

cudaError_t launch_silu_mul(const float *gu, int T, int F, float *out, long long ld_out, int num_sms, cudaStream_t st)
{
    if (T < 1 || F < 1 || ld_out < F) return cudaErrorInvalidValue;
    const long long n = (long long)T * F;
    long long blocks = (n + 255) / 256;
    if (blocks > 8LL * num_sms) blocks = 8LL * num_sms;
    return launch_pdl(silu_mul_kernel, dim3((unsigned)blocks), dim3(256), 0, st, gu, T, F, out, ld_out);
}

// out[i] = bf16(x[i]) (round to nearest even), n values, 8 per thread-step
// with 16-byte stores: the activation operand of the tensor-core matmul.
__global__ void f32_to_bf16_kernel(const float *__restrict__ x, long long n, __nv_bfloat16 *__restrict__ out)
{
    const long long n8 = n / 8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(x) + 2 * i);
        const float4 b = __ldg(reinterpret_cast<const float4 *>(x) + 2 * i + 1);
        __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y), p1 = __floats2bfloat162_rn(a.z, a.w);
        __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y), p3 = __floats2bfloat162_rn(b.z, b.w);
        uint4 o;
        o.x = *reinterpret_cast<uint32_t *>(&p0);
        o.y = *reinterpret_cast<uint32_t *>(&p1);
        o.z = *reinterpret_cast<uint32_t *>(&p2);
        o.w = *reinterpret_cast<uint32_t *>(&p3);
        reinterpret_cast<uint4 *>(out)[i] = o;
    }
    for (long long i = n8 * 8 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        out[i] = __float2bfloat16_rn(x[i]);
}

cudaError_t launch_f32_to_bf16(const float *x, long long n, __nv_bfloat16 *out, int num_sms, cudaStream_t st)
{
    if (n < 1 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
        return cudaErrorInvalidValue;
    long long blocks = (n / 8 + 255) / 256;
    if (blocks < 1) blocks = 1;
    if (blocks > 8LL * num_sms) blocks = 8LL * num_sms;
    f32_to_bf16_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, n, out);
    return cudaGetLastError();
}

} // namespace b200q
