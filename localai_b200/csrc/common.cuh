// Shared device helpers for the B200 GGML block-quant library (sm_100a).
//
// Block layouts (bytes per block / values per block) follow the GGML formats
// the reference decodes in engine/dequant.py:6-9:
//   Q4_0 18/32, Q8_0 34/32, Q4_K 144/256, Q5_K 176/256, Q6_K 210/256.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace b200q {

enum : int { T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };

// Error codes written to the per-device error word by kernels.
enum : int {
    ERR_NONE = 0,
    ERR_WAIT_TIMEOUT = 1,     // an mbarrier wait exceeded its time limit
    ERR_BAD_INDEX = 2,        // a routing index or offset out of range
};

template <int T> struct Fmt;
template <> struct Fmt<T_Q4_0> { static constexpr int VALS = 32,  BYTES = 18,  UPB = 1; };
template <> struct Fmt<T_Q8_0> { static constexpr int VALS = 32,  BYTES = 34,  UPB = 1; };
template <> struct Fmt<T_Q4_K> { static constexpr int VALS = 256, BYTES = 144, UPB = 8; };
template <> struct Fmt<T_Q5_K> { static constexpr int VALS = 256, BYTES = 176, UPB = 8; };
template <> struct Fmt<T_Q6_K> { static constexpr int VALS = 256, BYTES = 210, UPB = 8; };

__host__ __device__ inline int type_vals(int t) { return (t == T_Q4_K || t == T_Q5_K || t == T_Q6_K) ? 256 : 32; }
__host__ __device__ inline int type_bytes(int t)
{
    return t == T_Q4_0 ? 18 : t == T_Q8_0 ? 34 : t == T_Q4_K ? 144 : t == T_Q5_K ? 176 : t == T_Q6_K ? 210 : 0;
}

// fp16 bit pattern -> f32.  The hardware conversion is exact, subnormals
// included, matching half_to_float in native_quant.cpp:12-33.
__device__ __forceinline__ float h2f(uint32_t bits16)
{
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// A waiting warp is suspended in hardware until the phase completes or the
// hint (ns) runs out, instead of spinning: spinning warps compete with the
// producers and the MMA issuer for the barrier unit and for issue slots.
#ifndef MBAR_SUSPEND_NS
#define MBAR_SUSPEND_NS 1000000u
#endif
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(MBAR_SUSPEND_NS)
        : "memory");
    return ok != 0;
}

// Default limit for every device-side wait: 2 s.  A healthy wait here lasts
// microseconds; the limit exists so that a logic error ends the kernel with an
// error status instead of hanging a shared GPU.
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;

// Bounded wait on phase ``parity`` of an mbarrier.  On timeout it records
// ERR_WAIT_TIMEOUT in ``*err`` and returns false; callers then stop issuing
// work and leave.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int *err)
{
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > WAIT_LIMIT_NS) {
            atomicExch(err, ERR_WAIT_TIMEOUT);
            return false;
        }
    }
}

// Non-tensor bulk copy global -> shared, completing on an mbarrier.  Both
// addresses 16-byte aligned; size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch (kernels launched with the
// programmatic-stream-serialization attribute): let the next kernel of the
// stream start launching, and wait for the previous kernel's completion (and
// memory flush) before touching anything it may write.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Entry of every small kernel on the decode chain: the next kernel (usually a
// GEMV that starts streaming its constant weights at once) may launch now,
// and nothing of the previous kernel is read before it has completed.  Every
// kernel waits before it can complete, so completion stays transitive along
// the stream.
__device__ __forceinline__ void pdl_enter()
{
    pdl_launch_dependents();
    pdl_wait();
}

// Launch with programmatic stream serialization (the kernel may start while
// the previous kernel of the stream is still running; see pdl_enter).
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                     Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// silu(g) * u with silu(g) = g / (1 + exp(-clip(g, -80, 80)))
// (engine/model.py:161-166; the clip only keeps exp finite).
__device__ __forceinline__ float silu_mul(float g, float u)
{
    const float c = fminf(fmaxf(g, -80.f), 80.f);
    return g / (1.0f + expf(-c)) * u;
}

__device__ __forceinline__ void named_bar_sync(int id, int threads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Q4_K/Q5_K: the four 6-bit fields (scale, scale, min, min) of sub-blocks
// 2p and 2p+1 packed into bytes (engine/dequant.py:108-113).
__device__ __forceinline__ uint32_t k_scales_packed(const uint4 hdr, int p)
{
    const bool hk = p >= 2;
    const uint32_t i0 = (2 * p) & 3;
    const uint32_t sel = i0 | ((i0 + 1) << 4) | ((i0 + 4) << 8) | ((i0 + 5) << 12);
    const uint32_t lowsrc = __byte_perm(hk ? hdr.w : hdr.y, hk ? hdr.w : hdr.z, sel);
    const uint32_t lo4 = (lowsrc & 0x00000F0Fu) | ((lowsrc >> (hk ? 4 : 0)) & 0x0F0F0000u);
    const uint32_t top = __byte_perm(hdr.y, hdr.z, sel);
    return lo4 | ((top >> (hk ? 2 : 0)) & 0x30303030u);
}

// ---------------------------------------------------------------- shared loads
__device__ __forceinline__ uint32_t lds32(uint32_t a)
{
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a)
{
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a)
{
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t a)
{
    unsigned short v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}

// 16 bytes starting at any shared address (reads up to 4 bytes past the end).
template <bool ALIGNED16>
__device__ __forceinline__ uint4 lds128_any(uint32_t a)
{
    if (ALIGNED16) return lds128(a);
    const uint32_t base = a & ~3u;
    const uint32_t sh = (a & 3u) * 8u;
    const uint32_t w0 = lds32(base), w1 = lds32(base + 4), w2 = lds32(base + 8), w3 = lds32(base + 12),
                   w4 = lds32(base + 16);
    uint4 r;
    r.x = __funnelshift_r(w0, w1, sh);
    r.y = __funnelshift_r(w1, w2, sh);
    r.z = __funnelshift_r(w2, w3, sh);
    r.w = __funnelshift_r(w3, w4, sh);
    return r;
}

} // namespace b200q
