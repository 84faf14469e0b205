// Tensor-parallel exchange over NVLink / NVSwitch peer memory.
//
// Every rank owns one exchange region in its own HBM, exported to the other
// ranks through CUDA IPC; all regions share one layout, so a peer's field is
// the peer's base plus the same offset. Cross-GPU traffic is plain stores
// into the destination's region; the destination polls its own (local)
// memory. No TMA, no multicast, no library collective, no memory fences.
//
// Messages are "tagged words": every fp32 value travels in one 64-bit store
// together with a 32-bit tag, so a reader that sees the tag it expects also
// sees the value (a naturally aligned 64-bit access is single-copy atomic).
// Tag = frame * 256 + seq: `frame` is the step record's frame sequence number
// (advanced by the host for every frame, by the chained lm_head on the
// device), `seq` numbers the exchanges within a frame (2*layer + 0/1 for the
// two all-reduces of a layer, 255 for the greedy-id exchange). Every rank
// runs the same frames, so tags agree without host communication, and a tag
// is never reused, so stale words can never match.
//
//   recv    [2 slots][MF_TP_MAX senders][max_floats] u64   all-reduce partials (slot = seq & 1)
//   best    [MF_TP_MAX][2] u64                             per-rank lm_head maximum: value, index
//   gather  [gather_floats] f32                            full logits (each rank writes its slice)
//   local   CommLocal                                      this rank only: status
//   flags   [MF_TP_MAX] u64                                batched-prefill exchange: sender's epoch
//   bulk    [2 slots][bulk_floats] f32                     batched-prefill partials [rows][d]
//
// Batched prefill exchanges whole [rows, d] partials: each rank's GEMM writes
// its partial into its own bulk slot, the exchange kernel raises this rank's
// flag (a monotonic epoch) in every rank's region and, once every rank's flag
// shows the epoch, adds all ranks' slots in rank order. Slots alternate; a
// rank writes a slot again only after its next exchange, which needs every
// rank's flag for that exchange, raised after that rank finished reading.
//
// Slot reuse: consecutive all-reduces alternate slots. A rank cannot send
// into a slot again before every rank has read that slot's previous message:
// its next send there follows its receive of the other slot, which needs
// every rank's send of the other slot, which each rank issues only after its
// own receive of this slot.
//
// A wait is bounded by a wall-clock limit; on giving up it sets a status bit
// and the kernel carries on (its result is then garbage): nothing hangs.
#pragma once

#include "mf_common.cuh"

namespace mf {

constexpr int TP_MAX = MF_TP_MAX;
constexpr int COMM_STATUS_AR_TIMEOUT = 1;
constexpr int COMM_STATUS_LM_TIMEOUT = 2;
constexpr int COMM_SEQ_GREEDY = 255;

struct CommLocal {
    int status;  // COMM_STATUS_* bits; cleared by the host
    int pad[15];
    // arrival counters of the receiving kernels' grid barrier, per slot:
    // (tag << 32) | CTAs arrived (see grid_arrive_wait)
    unsigned long long bar[2];
    unsigned long long pad2[6];
};

struct CommLayout {
    size_t recv, best, gather, local, flags, bulk, total;
};

__host__ __device__ inline size_t comm_align(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline CommLayout comm_layout(int max_floats, int gather_floats, size_t bulk_floats = 0) {
    CommLayout L;
    L.recv = 0;
    L.best = comm_align(L.recv + (size_t)2 * TP_MAX * max_floats * 8, 256);
    L.gather = comm_align(L.best + (size_t)TP_MAX * 2 * 8, 256);
    L.local = comm_align(L.gather + (size_t)gather_floats * sizeof(float), 256);
    L.flags = comm_align(L.local + sizeof(CommLocal), 256);
    L.bulk = comm_align(L.flags + (size_t)TP_MAX * 8, 256);
    L.total = comm_align(L.bulk + 2 * bulk_floats * sizeof(float), 256);
    return L;
}

// Passed by value to kernels.
struct CommDev {
    char* base[TP_MAX];  // exchange region of every rank, mapped into this process
    int tp_rank, tp_size;
    int max_floats, gather_floats;
    unsigned long long timeout_ns;  // how long a wait polls before it gives up
    uint32_t off_recv, off_best, off_gather, off_local, off_flags, off_bulk;
    size_t bulk_floats;

    MF_DEVICE unsigned long long* recv(int owner, int slot, int sender) const {
        return reinterpret_cast<unsigned long long*>(base[owner] + off_recv) +
               ((size_t)slot * TP_MAX + sender) * max_floats;
    }
    MF_DEVICE unsigned long long* best(int owner) const {
        return reinterpret_cast<unsigned long long*>(base[owner] + off_best);
    }
    MF_DEVICE float* gather(int owner) const { return reinterpret_cast<float*>(base[owner] + off_gather); }
    MF_DEVICE CommLocal* local() const { return reinterpret_cast<CommLocal*>(base[tp_rank] + off_local); }
    MF_DEVICE unsigned long long* flags(int owner) const {
        return reinterpret_cast<unsigned long long*>(base[owner] + off_flags);
    }
    MF_DEVICE float* bulk(int owner, int slot) const {
        return reinterpret_cast<float*>(base[owner] + off_bulk) + (size_t)slot * bulk_floats;
    }
};

MF_DEVICE uint32_t comm_tag(int frame, int seq) { return (uint32_t)frame * 256u + (uint32_t)seq; }

MF_DEVICE unsigned long long tagged(float v, uint32_t tag) {
    return ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
}
MF_DEVICE void st_tagged(unsigned long long* p, unsigned long long w) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
MF_DEVICE unsigned long long ld_tagged(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

constexpr long long COMM_MAX_POLLS = 1ll << 26;  // backstop: the time limit ends a wait first

// Reads the tagged word at p once its tag is `tag`. Polls until `deadline`
// (globaltimer ns; and at most COMM_MAX_POLLS polls); after that, or when an
// earlier wait of the caller already gave up (*late), it sets `bit` in
// *status and returns whatever value is there.
MF_DEVICE float recv_tagged(const unsigned long long* p, uint32_t tag, unsigned long long deadline, bool* late,
                            int* status, int bit) {
    unsigned long long w = ld_tagged(p);
    if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
    if (!*late) {
        for (long long i = 0; i < COMM_MAX_POLLS; ++i) {
            __nanosleep(32);
            w = ld_tagged(p);
            if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
            if (globaltimer_ns() > deadline) break;
        }
        *late = true;
        atomicOr(status, bit);
    }
    return __uint_as_float((uint32_t)w);
}

// Grid barrier of one receiving kernel, on a counter word holding
// (tag << 32) | arrivals: the first CTA of this exchange replaces a stale tag
// (compare-and-swap), the others add one; then every CTA polls until all
// `n_ctas` have arrived. Every CTA of the grid is resident (the grid is sized
// to the SMs' capacity, and the dependent kernel launches only after all of
// this grid's CTAs started), so the barrier completes; it is bounded by
// `deadline` all the same (then it sets `bit` in *status and returns). The
// slot is reused two exchanges later, after this kernel completed. Called by
// one thread per CTA, after the CTA's writes were fenced.
MF_DEVICE void grid_arrive_wait(unsigned long long* ctr, uint32_t tag, unsigned n_ctas, unsigned long long deadline,
                                bool* late, int* status, int bit) {
    unsigned long long old;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(old) : "l"(ctr) : "memory");
    for (;;) {
        if ((uint32_t)(old >> 32) == tag) {
            atomicAdd(ctr, 1ull);
            break;
        }
        const unsigned long long prev = atomicCAS(ctr, old, ((unsigned long long)tag << 32) | 1ull);
        if (prev == old) break;
        old = prev;
    }
    const unsigned long long target = ((unsigned long long)tag << 32) | n_ctas;
    for (long long i = 0; i < COMM_MAX_POLLS; ++i) {
        unsigned long long v;
        asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(ctr) : "memory");
        if (v == target) return;
        if (*late || globaltimer_ns() > deadline) break;
        __nanosleep(20);
    }
    *late = true;
    atomicOr(status, bit);
}

// x[i] = x_res[i] + partial_0[i] + ... + partial_{tp-1}[i] (rank order) for
// the elements i = i0, i0 + stride, ... (< n) handled by one thread; all the
// partial words of a batch are loaded before any is checked, so a thread has
// COMM_WORDS_IN_FLIGHT tagged loads outstanding. Calls f(i, x[i]).
constexpr int COMM_WORDS_IN_FLIGHT = 16;

template <int TP, typename F>
MF_DEVICE void recv_sum_tp(const CommDev& c, int slot, uint32_t tag, const float* x_res, int i0, int stride, int n,
                           unsigned long long deadline, bool* late, int* status, F& f) {
    constexpr int RB = COMM_WORDS_IN_FLIGHT / TP;  // elements per batch
    for (int ib = i0; ib < n; ib += stride * RB) {
        unsigned long long w[TP][RB];
#pragma unroll
        for (int r = 0; r < TP; ++r)
#pragma unroll
            for (int b = 0; b < RB; ++b) {
                const int i = ib + b * stride;
                w[r][b] = i < n ? ld_tagged(c.recv(c.tp_rank, slot, r) + i) : 0ull;
            }
#pragma unroll
        for (int b = 0; b < RB; ++b) {
            const int i = ib + b * stride;
            if (i < n) {
                float v = __ldcg(x_res + i);
#pragma unroll
                for (int r = 0; r < TP; ++r)
                    v += ((uint32_t)(w[r][b] >> 32) == tag)
                             ? __uint_as_float((uint32_t)w[r][b])
                             : recv_tagged(c.recv(c.tp_rank, slot, r) + i, tag, deadline, late, status,
                                           COMM_STATUS_AR_TIMEOUT);
                f(i, v);
            }
        }
    }
}

template <typename F>
MF_DEVICE void recv_sum(const CommDev& c, int slot, uint32_t tag, const float* x_res, int i0, int stride, int n,
                        unsigned long long deadline, bool* late, int* status, F&& f) {
    switch (c.tp_size) {
        case 1: recv_sum_tp<1>(c, slot, tag, x_res, i0, stride, n, deadline, late, status, f); break;
        case 2: recv_sum_tp<2>(c, slot, tag, x_res, i0, stride, n, deadline, late, status, f); break;
        case 4: recv_sum_tp<4>(c, slot, tag, x_res, i0, stride, n, deadline, late, status, f); break;
        case 8: recv_sum_tp<8>(c, slot, tag, x_res, i0, stride, n, deadline, late, status, f); break;
        default:  // 3, 5, 6, 7 ranks: one element at a time
            for (int i = i0; i < n; i += stride) {
                float v = __ldcg(x_res + i);
                for (int r = 0; r < c.tp_size; ++r)
                    v += recv_tagged(c.recv(c.tp_rank, slot, r) + i, tag, deadline, late, status,
                                     COMM_STATUS_AR_TIMEOUT);
                f(i, v);
            }
    }
}

}  // namespace mf
