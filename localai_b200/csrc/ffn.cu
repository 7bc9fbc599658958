// Dense FFN glue for the decode path (engine/model.py:161-166, :230-233):
//   act[t, f] = silu(gate[t, f]) * up[t, f],  silu(g) = g / (1 + exp(-clip(g, -80, 80)))
// (act rows ld_out apart, so a zero-padded K tail can follow the F values)
// with gate and up read from one [T, 2F] f32 matrix (the output of a single
// GEMV over the concatenated [gate; up] weights).  HBM-bound elementwise.
#include "common.cuh"

namespace b200q {

__global__ void silu_mul_kernel(const float *__restrict__ gu, int T, int F, float *__restrict__ out, long long ld_out)
{
    const long long n = (long long)T * F;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / F;
        const int f = (int)(i - t * F);
        const float g = gu[t * 2 * F + f], u = gu[t * 2 * F + F + f];
        const float c = fminf(fmaxf(g, -80.f), 80.f);
        out[t * ld_out + f] = g / (1.0f + expf(-c)) * u;
    }
}

cudaError_t launch_silu_mul(const float *gu, int T, int F, float *out, long long ld_out, int num_sms, cudaStream_t st)
{
    if (T < 1 || F < 1 || ld_out < F) return cudaErrorInvalidValue;
    const long long n = (long long)T * F;
    long long blocks = (n + 255) / 256;
    if (blocks > 8LL * num_sms) blocks = 8LL * num_sms;
    silu_mul_kernel<<<(int)blocks, 256, 0, st>>>(gu, T, F, out, ld_out);
    return cudaGetLastError();
}

} // namespace b200q
