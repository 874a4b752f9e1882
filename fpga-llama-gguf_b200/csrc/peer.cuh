// Device side of the row-sharded passes without a collective (PeerSync / PeerWait in kernel_args.h): stores into
// the peers' act over NVLink (plain stores to IPC-mapped memory), the ready / data words, and their bounded waits.
#pragma once
#include "kernel_args.h"
#include "pipeline.cuh"

namespace b200q {

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// count v has reached k (counts only grow, modulo 2^32)
__device__ __forceinline__ bool reached(unsigned v, unsigned k) { return int(v - k) >= 0; }

// Bounded wait until *p reaches k; false on timeout.
__device__ __forceinline__ bool wait_reached(const unsigned *p, unsigned k) {
    unsigned long long t0 = 0;
    for (unsigned i = 0; !reached(ld_acquire_sys(p), k); ++i) {
        if ((i & 255u) == 255u) {
            const unsigned long long now = global_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > kWaitLimitNs) return false;
        }
    }
    return true;
}

// Store v at p in this rank's act and at the same offset in every peer's act.
__device__ __forceinline__ void peer_store(const PeerSync *ps, float *p, float v) {
    *p = v;
    if (ps) {
        const size_t off = size_t(p - ps->act);
#pragma unroll 1
        for (unsigned r = 0; r < ps->world; ++r)
            if (ps->peer_act[r]) ps->peer_act[r][off] = v;
    }
}

// the number of this launch among the slot's launches (1, 2, ...)
__device__ __forceinline__ unsigned launch_number(const PeerSync &ps) { return ps.sync[kSyncMineWord + ps.slot] + 1u; }

// This rank has reached the launch (once per launch, after the wait on the previous kernel).
__device__ __forceinline__ void peer_announce(const PeerSync &ps) {
    const unsigned k = launch_number(ps);
    for (unsigned r = 0; r < ps.world; ++r)
        if (ps.peer_sync[r]) st_release_sys(ps.peer_sync[r] + ready_word(ps.slot, ps.rank), k);
}

// Bounded wait until every peer has reached the launch (before the first store into a peer); false on timeout.
__device__ __forceinline__ bool peer_wait_ready(const PeerSync &ps) {
    const unsigned k = launch_number(ps);
    bool ok = true;
    for (unsigned r = 0; r < ps.world; ++r)
        if (r != ps.rank) ok = wait_reached(ps.sync + ready_word(ps.slot, r), k) && ok;
    return ok;
}

// One thread per CTA, after the threads that stored into peers synchronised with it: count the CTA with a
// system-scope acquire-release add (its rows in the peers become visible before the count); the last CTA, which has
// acquired every other CTA's count, raises its data word in every peer (release), re-arms the CTA counter and counts
// the launch. (One system-scope fence per thread instead cost ~15 us per pass.)
__device__ __forceinline__ void peer_signal(const PeerSync &ps, unsigned ctas) {
    unsigned prev;
    asm volatile("atom.acq_rel.sys.global.add.u32 %0, [%1], 1;"
                 : "=r"(prev)
                 : "l"(ps.sync + kSyncCountWord + ps.slot)
                 : "memory");
    if (prev == ctas - 1) {
        ps.sync[kSyncCountWord + ps.slot] = 0;
        const unsigned k = launch_number(ps);
        for (unsigned r = 0; r < ps.world; ++r)
            if (ps.peer_sync[r]) st_release_sys(ps.peer_sync[r] + data_word(ps.slot, ps.rank), k);
        ps.sync[kSyncMineWord + ps.slot] = k;
    }
}

// One thread: bounded wait until every peer's data word of each slot of pw reached this rank's own launch count of
// that slot (this rank's launch has completed: the kernel runs after it). On timeout the error word is set.
__device__ __forceinline__ void peer_wait_rows(const PeerWait &pw) {
    for (unsigned i = 0; i < pw.n; ++i) {
        const unsigned slot = pw.slot0 + i, k = pw.sync[kSyncMineWord + slot];
        for (unsigned r = 0; r < pw.world; ++r) {
            if (r == pw.rank) continue;
            if (!wait_reached(pw.sync + data_word(slot, r), k)) {
                if (pw.err) atomicExch(pw.err, 1u);
                return;
            }
        }
    }
}

// Whole CTA: thread 0 waits, then the CTA proceeds (call after pdl_wait, before reading act).
__device__ __forceinline__ void peer_wait_rows_cta(const PeerWait &pw) {
    if (pw.n) {
        if (threadIdx.x == 0) peer_wait_rows(pw);
        __syncthreads();
    }
}

}  // namespace b200q
