// Expert-parallel exchange over peer memory (one process per GPU, NVLink /
// NVSwitch, CUDA IPC mappings of each rank's exchange region).
//
// Each rank owns one exchange region, mapped by every other rank:
//   [EpShared header | recv rows bf16 [cap_recv, D] | return rows bf16 [cap_send, D]]
// Receive rows are expert-major; inside an expert's group the runs of the
// sources follow the order me, me+1, ... (the receiver's own rows first).
// Senders write straight into the receiver's region (plain stores through the
// peer mapping; no TMA, no multicast) and raise per-source flags with release
// stores at system scope; receivers poll their own flags with acquire loads
// under a time limit.  Flags carry the call's epoch (1, 2, ...), so nothing
// is ever reset between calls.
#pragma once
#include "common.cuh"
#include <cstdint>
#include <cuda_bf16.h>

namespace b200q {

constexpr int EP_MAX_RANKS = 8;
constexpr int EP_MAX_EXPERTS = 256;     // G * experts-per-rank
// Fused exchange: every receiver's rows are cut into GEMM row tiles of
// EP_TILE_ROWS (group by group) and the tiles into rounds: a first round of
// at most EP_FIRST_ROUND tiles (about what the GEMM's first wave of tiles
// reads), then rounds of rt tiles, at most EP_ROUNDS_TARGET + 2 in all; a
// source announces each round once its rows of that round have landed at
// every receiver.
constexpr int EP_TILE_ROWS = 256;
constexpr int EP_ROUNDS_TARGET = 16;
constexpr int EP_FIRST_ROUND = 8;
constexpr int EP_MAX_ROUNDS = 32;

// Round of row tile q (EpDev::r0, rt) and first tile of round r.
__host__ __device__ inline int ep_round_of_tile(int q, int r0, int rt) { return q < r0 ? 0 : 1 + (q - r0) / rt; }
__host__ __device__ inline int ep_round_first_tile(int r, int r0, int rt) { return r == 0 ? 0 : r0 + (r - 1) * rt; }

struct EpShared {
    uint32_t cnt_flag[EP_MAX_RANKS];    // source s's routing counts have arrived
    uint32_t row_flag[EP_MAX_RANKS];    // source s's rows have arrived
    uint32_t ret_flag[EP_MAX_RANKS];    // owner s has written my expert outputs back
    uint32_t pad[64 - 3 * EP_MAX_RANKS];
    int inbox[EP_MAX_RANKS][EP_MAX_EXPERTS];   // [source][virtual expert] row counts
    // dispatch fused into the gate/up GEMM: round_flag[s][r] = epoch once
    // source s has stored every row it sends for my row tiles of round r
    uint32_t round_flag[EP_MAX_RANKS][EP_MAX_ROUNDS];
};

// Device-resident tables of one rank (not shared).
struct EpDev {
    EpShared *peer_shared[EP_MAX_RANKS];
    __nv_bfloat16 *peer_recv[EP_MAX_RANKS];
    __nv_bfloat16 *peer_ret[EP_MAX_RANKS];
    int G, me, E_loc, D;
    long long cap_recv, cap_send;
    unsigned int done;                        // CTAs of the send kernel that finished
    unsigned int round_done[EP_MAX_ROUNDS];   // fused dispatch: push warps done with round r
    uint32_t epoch;                           // epoch of the current call (device-side counter)
    int blocked;                              // bit d: rank d's receive buffer would overflow
    // Receive layout (expert-major; within a group the sources in the order
    // me, me+1, ...), rebuilt by every count exchange:
    int grp_off[EP_MAX_EXPERTS + 1];          // [E_loc + 1] rows of local expert e start here
    int run_off[EP_MAX_EXPERTS + 1];          // [e * G + j] rows from source (me + j) % G for expert e
    int ret_base[EP_MAX_EXPERTS];             // [e * G + j] first slot of that run in its source's slot order
    // Send layout: rows of my virtual expert v = d * E_loc + e start at dst_off[v]
    // in rank d's receive buffer.
    int dst_off[EP_MAX_EXPERTS];
    // Every rank's receive layout, for the fused exchange's rounds: rank d's
    // group g (local expert) starts at row dgrp_off[d * (E_loc + 1) + g] and at
    // row tile dtile[d * (E_loc + 1) + g] (tiles of EP_TILE_ROWS, group by
    // group); round 0 is tiles [0, r0), round r > 0 tiles
    // [r0 + (r-1) rt, r0 + r rt); ``rounds`` covers the largest layout.
    int dgrp_off[EP_MAX_EXPERTS + EP_MAX_RANKS];
    int dtile[EP_MAX_EXPERTS + EP_MAX_RANKS];
    int r0, rt, rounds;
};

// Expert-parallel dispatch fused into the gate/up grouped GEMM: while the
// GEMM runs, one warp of every CTA stores this rank's routed rows into their
// owners' receive buffers, round by round of the receivers' row tiles, and
// each GEMM tile waits only for its own round (round_flag) instead of for the
// whole exchange.
struct EpPush {
    const EpDev *ep;            // this rank's device tables
    const __nv_bfloat16 *h;     // bf16 [T, D] token rows (the router's copy of h)
    const int *token_of;        // [S] token of each routed slot, dispatch (virtual expert) order
    const int *offsets;         // [G * E_loc + 1] first slot of each virtual expert
    int S, T;
    uint32_t epoch;             // 0: the device-side counter
    unsigned long long wait_ns; // limit of each wait on a peer's flag
};

#ifdef __CUDACC__
__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait until *flag has reached ``epoch`` (wrap-safe comparison), for at most
// limit_ns nanoseconds (and 2^30 polls); on time-out the error word is set.
__device__ __forceinline__ bool ep_wait_flag(const uint32_t *flag, uint32_t epoch, int *err, uint64_t limit_ns)
{
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 0;; ++it) {
        if ((int)(ld_acquire_sys(flag) - epoch) >= 0) return true;
        if ((it & 63) == 63 && (global_timer_ns() - t0 > limit_ns || it > (1u << 30))) {
            atomicExch(err, ERR_WAIT_TIMEOUT);
            return false;
        }
        __nanosleep(100);
    }
}
#endif

unsigned long long ep_wait_ns();

} // namespace b200q
