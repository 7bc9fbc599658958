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

} // namespace b200q
