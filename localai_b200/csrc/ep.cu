// Expert-parallel exchange kernels over NVLink peer memory (see ep.cuh).
//
// One forward of the expert-parallel MoE layer on rank ``me`` of G:
//   ep_counts_kernel   write my per-(rank, expert) row counts into every
//                      rank's inbox, raise cnt_flag there, wait for all G
//                      inboxes, then build the receive and send layouts;
//   ep_send_kernel     gather my routed rows (f32 -> bf16) and store each one
//                      directly into its owner's receive buffer (expert-major;
//                      in a group the owner's own rows first, then ranks
//                      owner+1, ...), then raise row_flag at every rank;
//   ep_wait_kernel     wait for row_flag (before the GEMMs) or ret_flag
//                      (before the combine) from all G ranks;
//   (gate/up GEMM on the received rows; down GEMM whose epilogue stores each
//    output row straight into the source rank's return buffer)
//   ep_signal_kernel   raise ret_flag at every rank.
// All waits are bounded (g_ep_wait_ns); a wait that runs out sets the device
// error word and the kernel returns, so the host sees an error instead of a
// hang.
//
// Epochs: an epoch argument of 0 means "the device-side counter": the count
// exchange advances it (ep->epoch + 1) and the later kernels of the call read
// it, so a whole layer call can be captured once in a CUDA graph and
// replayed.  A nonzero argument is used as given (and stored as the counter).
#include "common.cuh"
#include "ep.cuh"

#include <cstring>

namespace b200q {

// Time limit of every wait on another rank's flag (default 5 s), settable
// with b200q_ep_set_wait_limit_ns; passed to each waiting kernel at launch.
static unsigned long long g_ep_wait_ns = 5000000000ull;
void ep_set_wait_ns(unsigned long long ns) { g_ep_wait_ns = ns ? ns : 5000000000ull; }
unsigned long long ep_wait_ns() { return g_ep_wait_ns; }

__global__ void __launch_bounds__(256) ep_counts_kernel(EpDev *ep, const int *__restrict__ offsets, uint32_t epoch,
                                                        int *err, uint64_t limit_ns)
{
    __shared__ int cnt[EP_MAX_RANKS][EP_MAX_EXPERTS];
    __shared__ int ok_s, blocked_s;
    const int tid = threadIdx.x;
    const int G = ep->G, me = ep->me, El = ep->E_loc, E = G * El;
    EpShared *mine = ep->peer_shared[me];
    epoch = epoch ? epoch : ep->epoch + 1;           // every thread reads the counter before it is advanced
    for (int v = tid; v < E; v += blockDim.x) {
        const int c = offsets[v + 1] - offsets[v];
        for (int d = 0; d < G; ++d) ep->peer_shared[d]->inbox[me][v] = c;
    }
    for (int r = tid; r < EP_MAX_ROUNDS; r += blockDim.x) ep->round_done[r] = 0;
    if (tid == 0) {
        ep->done = 0;
        ok_s = 1;
        blocked_s = 0;
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) ep->epoch = epoch;
    if (tid < G) st_release_sys(&ep->peer_shared[tid]->cnt_flag[me], epoch);
    if (tid < G && !ep_wait_flag(&mine->cnt_flag[tid], epoch, err, limit_ns)) ok_s = 0;
    __syncthreads();
    if (!ok_s) {
        // no layout: send nothing, receive nothing
        for (int i = tid; i <= El; i += blockDim.x) ep->grp_off[i] = 0;
        for (int i = tid; i <= E; i += blockDim.x) ep->run_off[i] = 0;
        if (tid == 0) {
            ep->blocked = (1 << G) - 1;
            ep->rounds = 0;
            ep->rt = 1;
            ep->r0 = 1;
        }
        return;
    }
    for (int i = tid; i < G * E; i += blockDim.x) cnt[i / E][i % E] = __ldcg(&mine->inbox[i / E][i % E]);
    __syncthreads();
    // rows each rank d would receive; a rank whose buffer would overflow gets nothing
    if (tid < G) {
        long long tot = 0;
        for (int s = 0; s < G; ++s)
            for (int e = 0; e < El; ++e) tot += cnt[s][tid * El + e];
        if (tot > ep->cap_recv) {
            atomicOr(&blocked_s, 1 << tid);
            atomicExch(err, ERR_BAD_INDEX);
        }
    }
    __syncthreads();
    const bool me_blocked = (blocked_s >> me) & 1;
    const int vme = me * El;
    for (int i = tid; i < E; i += blockDim.x) {
        // receive runs: i = e * G + j, the j-th run of group e, from source
        // (me + j) % G -- every group starts with this rank's own rows, so that
        // the first row tiles of every rank are fed by local copies and the
        // sources' shares of a rank's early tiles rotate with the rank
        {
            const int e = i / G, j = i % G, s = (me + j) % G;
            int r = 0;
            for (int e2 = 0; e2 < e; ++e2)
                for (int s2 = 0; s2 < G; ++s2) r += cnt[s2][vme + e2];
            for (int j2 = 0; j2 < j; ++j2) r += cnt[(me + j2) % G][vme + e];
            ep->run_off[i] = me_blocked ? 0 : r;
            int b = 0;
            for (int v = 0; v < vme + e; ++v) b += cnt[s][v];
            ep->ret_base[i] = b;
        }
        // send runs: i = d * El + e (virtual expert): my run is the
        // ((me - d) mod G)-th of rank d's group e
        {
            const int d = i / El, e = i % El;
            int r = 0;
            for (int e2 = 0; e2 < e; ++e2)
                for (int s2 = 0; s2 < G; ++s2) r += cnt[s2][d * El + e2];
            for (int j2 = 0; j2 < (me - d + G) % G; ++j2) r += cnt[(d + j2) % G][i];
            ep->dst_off[i] = r;
        }
    }
    for (int e = tid; e <= El; e += blockDim.x) {
        int r = 0;
        for (int e2 = 0; e2 < e; ++e2)
            for (int s2 = 0; s2 < G; ++s2) r += cnt[s2][vme + e2];
        ep->grp_off[e] = me_blocked ? 0 : r;
        if (e == El) ep->run_off[E] = me_blocked ? 0 : r;
    }
    // every rank's group row offsets and row-tile bases (the fused exchange's
    // rounds); all ranks compute the same tables from the same counts
    if (tid < G) {
        const int d = tid;
        int rows = 0, tiles = 0;
        for (int g = 0; g <= El; ++g) {
            ep->dgrp_off[d * (El + 1) + g] = rows;
            ep->dtile[d * (El + 1) + g] = tiles;
            if (g == El) break;
            int m = 0;
            for (int s2 = 0; s2 < G; ++s2) m += cnt[s2][d * El + g];
            rows += m;
            tiles += (m + EP_TILE_ROWS - 1) / EP_TILE_ROWS;
        }
    }
    __syncthreads();
    if (tid == 0) {
        ep->blocked = blocked_s;
        int qmax = 0;
        for (int d = 0; d < G; ++d) qmax = max(qmax, ep->dtile[d * (El + 1) + El]);
        const int rt = max(1, (qmax + EP_ROUNDS_TARGET - 1) / EP_ROUNDS_TARGET);
        const int r0 = min(rt, EP_FIRST_ROUND);
        ep->rt = rt;
        ep->r0 = r0;
        // <= 1 + EP_ROUNDS_TARGET + 1 <= EP_MAX_ROUNDS
        ep->rounds = qmax == 0 ? 0 : qmax <= r0 ? 1 : 1 + (qmax - r0 + rt - 1) / rt;
    }
}

// Source rows f32 (converted to bf16 on the way) or already bf16 (the
// router's copy of h: a plain 16-byte copy, four loads in flight per lane).
template <typename TIn>
__global__ void __launch_bounds__(256) ep_send_kernel(EpDev *ep, const TIn *__restrict__ h,
                                                      const int *__restrict__ token_of,
                                                      const int *__restrict__ offsets, int S, int T, uint32_t epoch,
                                                      int *err)
{
    __shared__ int off_s[EP_MAX_EXPERTS + 1], dst_s[EP_MAX_EXPERTS];
    __shared__ __nv_bfloat16 *peer_s[EP_MAX_RANKS];
    __shared__ int blocked_s;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = ep->G, me = ep->me, El = ep->E_loc, E = G * El, D = ep->D;
    for (int i = tid; i <= E; i += blockDim.x) off_s[i] = offsets[i];
    for (int i = tid; i < E; i += blockDim.x) dst_s[i] = ep->dst_off[i];
    if (tid < G) peer_s[tid] = ep->peer_recv[tid];
    if (tid == 0) blocked_s = ep->blocked;
    __syncthreads();
    // slots at or past offsets[E] belong to pairs with a bad expert id: not sent
    const int n_valid = min(S, off_s[E]);
    // start with the rows for rank me + 1 (then me + 2, ...; my own last), so
    // that the ranks' first stores go to different destinations instead of
    // all of them filling rank 0's receive buffer first
    const int start = n_valid ? off_s[((me + 1) % G) * El] % n_valid : 0;
    for (int j = blockIdx.x * 8 + warp; j < n_valid; j += gridDim.x * 8) {
        const int i = j + start < n_valid ? j + start : j + start - n_valid;
        int lo = 0, hi = E;                          // largest v with off_s[v] <= i
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (off_s[mid] <= i) lo = mid; else hi = mid;
        }
        const int d = lo / El;
        if ((blocked_s >> d) & 1) continue;
        const int t = token_of[i];
        if (t < 0 || t >= T) {
            if (lane == 0) atomicExch(err, ERR_BAD_INDEX);
            continue;
        }
        __nv_bfloat16 *dst = peer_s[d] + (long long)(dst_s[lo] + (i - off_s[lo])) * D;
        if constexpr (sizeof(TIn) == 2) {
            const uint4 *src = reinterpret_cast<const uint4 *>(h + (long long)t * D);
            uint4 *d16 = reinterpret_cast<uint4 *>(dst);
            const int n = D / 8;
            int c = lane;
            for (; c + 96 < n; c += 128) {
                const uint4 v0 = __ldg(src + c), v1 = __ldg(src + c + 32), v2 = __ldg(src + c + 64),
                            v3 = __ldg(src + c + 96);
                d16[c] = v0;
                d16[c + 32] = v1;
                d16[c + 64] = v2;
                d16[c + 96] = v3;
            }
            for (; c < n; c += 32) d16[c] = __ldg(src + c);
            continue;
        }
        const float *src = reinterpret_cast<const float *>(h) + (long long)t * D;
        for (int c = lane * 8; c < D; c += 256) {
            const float4 a = __ldg(reinterpret_cast<const float4 *>(src + c));
            const float4 b = __ldg(reinterpret_cast<const float4 *>(src + c + 4));
            __nv_bfloat162 p0 = __floats2bfloat162_rn(a.x, a.y), p1 = __floats2bfloat162_rn(a.z, a.w);
            __nv_bfloat162 p2 = __floats2bfloat162_rn(b.x, b.y), p3 = __floats2bfloat162_rn(b.z, b.w);
            uint4 o;
            o.x = *reinterpret_cast<uint32_t *>(&p0);
            o.y = *reinterpret_cast<uint32_t *>(&p1);
            o.z = *reinterpret_cast<uint32_t *>(&p2);
            o.w = *reinterpret_cast<uint32_t *>(&p3);
            *reinterpret_cast<uint4 *>(dst + c) = o;
        }
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) {
        const unsigned old = atomicAdd(&ep->done, 1u);
        if (old == gridDim.x - 1) {
            __threadfence_system();
            const uint32_t e = epoch ? epoch : ep->epoch;
            for (int d = 0; d < G; ++d) st_release_sys(&ep->peer_shared[d]->row_flag[me], e);
        }
    }
}

// which: 1 = rows arrived from every rank, 2 = expert outputs returned by every rank.
__global__ void ep_wait_kernel(EpDev *ep, int which, uint32_t epoch, int *err, uint64_t limit_ns)
{
    const int lane = threadIdx.x;
    EpShared *mine = ep->peer_shared[ep->me];
    epoch = epoch ? epoch : ep->epoch;
    if (lane < ep->G) ep_wait_flag(which == 1 ? &mine->row_flag[lane] : &mine->ret_flag[lane], epoch, err, limit_ns);
}

__global__ void ep_signal_kernel(EpDev *ep, uint32_t epoch)
{
    __threadfence_system();
    const int lane = threadIdx.x;
    epoch = epoch ? epoch : ep->epoch;
    if (lane < ep->G) st_release_sys(&ep->peer_shared[lane]->ret_flag[ep->me], epoch);
}

// ---------------------------------------------------------------- host side
struct EpHost {
    int device = -1;
    int G = 0, me = 0, E_loc = 0, D = 0;
    long long cap_send = 0, cap_recv = 0;
    char *region = nullptr;
    size_t off_recv = 0, off_ret = 0, bytes = 0;
    void *peer_base[EP_MAX_RANKS] = {};
    EpDev *dev = nullptr;
    bool opened = false;
};

static size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

cudaError_t ep_create(int G, int me, int E_loc, int D, long long cap_send, long long cap_recv, void **out)
{
    *out = nullptr;
    if (G < 1 || G > EP_MAX_RANKS || me < 0 || me >= G || E_loc < 1 || G * E_loc > EP_MAX_EXPERTS || D < 8 ||
        D % 8 || cap_send < 1 || cap_recv < 1)
        return cudaErrorInvalidValue;
    EpHost *p = new EpHost;
    cudaGetDevice(&p->device);
    p->G = G;
    p->me = me;
    p->E_loc = E_loc;
    p->D = D;
    p->cap_send = cap_send;
    p->cap_recv = cap_recv;
    p->off_recv = align_up(sizeof(EpShared), 4096);
    p->off_ret = p->off_recv + align_up((size_t)cap_recv * D * 2, 4096);
    p->bytes = p->off_ret + align_up((size_t)cap_send * D * 2, 4096);
    cudaError_t e = cudaMalloc(&p->region, p->bytes);
    if (e == cudaSuccess) e = cudaMemset(p->region, 0, sizeof(EpShared));
    if (e == cudaSuccess) e = cudaMalloc(&p->dev, sizeof(EpDev));
    if (e == cudaSuccess) e = cudaMemset(p->dev, 0, sizeof(EpDev));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (p->region) cudaFree(p->region);
        if (p->dev) cudaFree(p->dev);
        delete p;
        return e;
    }
    *out = p;
    return cudaSuccess;
}

cudaError_t ep_ipc_handle(void *ctx, void *handle64)
{
    EpHost *p = static_cast<EpHost *>(ctx);
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, p->region);
    if (e == cudaSuccess) std::memcpy(handle64, &h, sizeof(h));
    return e;
}

size_t ep_ipc_handle_bytes() { return sizeof(cudaIpcMemHandle_t); }

cudaError_t ep_open(void *ctx, const void *handles)
{
    EpHost *p = static_cast<EpHost *>(ctx);
    if (p->opened) return cudaErrorInvalidValue;
    EpDev h;
    std::memset(&h, 0, sizeof(h));
    for (int s = 0; s < p->G; ++s) {
        char *base = nullptr;
        if (s == p->me) {
            base = p->region;
        } else {
            cudaIpcMemHandle_t mh;
            std::memcpy(&mh, static_cast<const char *>(handles) + s * sizeof(cudaIpcMemHandle_t), sizeof(mh));
            void *q = nullptr;
            cudaError_t e = cudaIpcOpenMemHandle(&q, mh, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) return e;
            p->peer_base[s] = q;
            base = static_cast<char *>(q);
        }
        h.peer_shared[s] = reinterpret_cast<EpShared *>(base);
        h.peer_recv[s] = reinterpret_cast<__nv_bfloat16 *>(base + p->off_recv);
        h.peer_ret[s] = reinterpret_cast<__nv_bfloat16 *>(base + p->off_ret);
    }
    h.G = p->G;
    h.me = p->me;
    h.E_loc = p->E_loc;
    h.D = p->D;
    h.cap_recv = p->cap_recv;
    h.cap_send = p->cap_send;
    cudaError_t e = cudaMemcpy(p->dev, &h, sizeof(h), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) p->opened = true;
    return e;
}

cudaError_t ep_destroy(void *ctx)
{
    EpHost *p = static_cast<EpHost *>(ctx);
    cudaError_t first = cudaDeviceSynchronize();
    for (int s = 0; s < p->G; ++s)
        if (p->peer_base[s]) {
            cudaError_t e = cudaIpcCloseMemHandle(p->peer_base[s]);
            if (first == cudaSuccess) first = e;
        }
    if (p->region) cudaFree(p->region);
    if (p->dev) cudaFree(p->dev);
    delete p;
    return first;
}

bool ep_is_open(void *ctx) { return static_cast<EpHost *>(ctx)->opened; }
void *ep_recv_rows(void *ctx) { EpHost *p = static_cast<EpHost *>(ctx); return p->region + p->off_recv; }
void *ep_ret_rows(void *ctx) { EpHost *p = static_cast<EpHost *>(ctx); return p->region + p->off_ret; }
EpDev *ep_dev(void *ctx) { return static_cast<EpHost *>(ctx)->dev; }
const int *ep_group_offsets(void *ctx) { return static_cast<EpHost *>(ctx)->dev->grp_off; }
long long ep_cap_recv(void *ctx) { return static_cast<EpHost *>(ctx)->cap_recv; }
long long ep_cap_send(void *ctx) { return static_cast<EpHost *>(ctx)->cap_send; }
int ep_local_experts(void *ctx) { return static_cast<EpHost *>(ctx)->E_loc; }
int ep_d_model(void *ctx) { return static_cast<EpHost *>(ctx)->D; }

cudaError_t launch_ep_counts(void *ctx, const int *offsets, uint32_t epoch, int *err, cudaStream_t st)
{
    EpHost *p = static_cast<EpHost *>(ctx);
    if (!p->opened) return cudaErrorInvalidValue;
    ep_counts_kernel<<<1, 256, 0, st>>>(p->dev, offsets, epoch, err, g_ep_wait_ns);
    return cudaGetLastError();
}

cudaError_t launch_ep_send(void *ctx, const void *h, bool h_bf16, const int *token_of, const int *offsets, int S,
                           int T, uint32_t epoch, int *err, int num_sms, cudaStream_t st)
{
    EpHost *p = static_cast<EpHost *>(ctx);
    if (!p->opened || S < 0 || (long long)S > p->cap_send || (reinterpret_cast<uintptr_t>(h) & 15))
        return cudaErrorInvalidValue;
    int grid = (S + 7) / 8;
    if (grid > num_sms * 8) grid = num_sms * 8;
    if (grid < 1) grid = 1;
    if (h_bf16)
        ep_send_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p->dev, static_cast<const __nv_bfloat16 *>(h), token_of,
                                                             offsets, S, T, epoch, err);
    else
        ep_send_kernel<float><<<grid, 256, 0, st>>>(p->dev, static_cast<const float *>(h), token_of, offsets, S, T,
                                                     epoch, err);
    return cudaGetLastError();
}

cudaError_t launch_ep_wait(void *ctx, int which, uint32_t epoch, int *err, cudaStream_t st)
{
    EpHost *p = static_cast<EpHost *>(ctx);
    if (!p->opened || (which != 1 && which != 2)) return cudaErrorInvalidValue;
    ep_wait_kernel<<<1, 32, 0, st>>>(p->dev, which, epoch, err, g_ep_wait_ns);
    return cudaGetLastError();
}

cudaError_t launch_ep_signal(void *ctx, uint32_t epoch, cudaStream_t st)
{
    EpHost *p = static_cast<EpHost *>(ctx);
    if (!p->opened) return cudaErrorInvalidValue;
    ep_signal_kernel<<<1, 32, 0, st>>>(p->dev, epoch);
    return cudaGetLastError();
}

} // namespace b200q
