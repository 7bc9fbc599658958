// Expert-parallel exchange over peer memory (one process per GPU, NVLink /
// NVSwitch, CUDA IPC mappings of each rank's exchange region).
//
// Each rank owns one exchange region, mapped by every other rank:
//   [EpShared header | recv rows bf16 [cap_recv, D] | return rows bf16 [cap_send, D]]
// Senders write straight into the receiver's region (plain stores through the
// peer mapping; no TMA, no multicast) and raise per-source flags with release
// stores at system scope; receivers poll their own flags with acquire loads
// under a time limit.  Flags carry the call's epoch (1, 2, ...), so nothing
// is ever reset between calls.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>

namespace b200q {

constexpr int EP_MAX_RANKS = 8;
constexpr int EP_MAX_EXPERTS = 256;     // G * experts-per-rank

struct EpShared {
    uint32_t cnt_flag[EP_MAX_RANKS];    // source s's routing counts have arrived
    uint32_t row_flag[EP_MAX_RANKS];    // source s's rows have arrived
    uint32_t ret_flag[EP_MAX_RANKS];    // owner s has written my expert outputs back
    uint32_t pad[64 - 3 * EP_MAX_RANKS];
    int inbox[EP_MAX_RANKS][EP_MAX_EXPERTS];   // [source][virtual expert] row counts
};

// Device-resident tables of one rank (not shared).
struct EpDev {
    EpShared *peer_shared[EP_MAX_RANKS];
    __nv_bfloat16 *peer_recv[EP_MAX_RANKS];
    __nv_bfloat16 *peer_ret[EP_MAX_RANKS];
    int G, me, E_loc, D;
    long long cap_recv, cap_send;
    unsigned int done;                        // CTAs of the send kernel that finished
    uint32_t epoch;                           // epoch of the current call (device-side counter)
    int blocked;                              // bit d: rank d's receive buffer would overflow
    // Receive layout (expert-major, source-minor), rebuilt by every count exchange:
    int grp_off[EP_MAX_EXPERTS + 1];          // [E_loc + 1] rows of local expert e start here
    int run_off[EP_MAX_EXPERTS + 1];          // [e * G + s] rows from source s for expert e
    int ret_base[EP_MAX_EXPERTS];             // [e * G + s] first slot of that run in s's slot order
    // Send layout: rows of my virtual expert v = d * E_loc + e start at dst_off[v]
    // in rank d's receive buffer.
    int dst_off[EP_MAX_EXPERTS];
};

} // namespace b200q
