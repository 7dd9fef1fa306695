// Expert parallelism over NVLink peer memory: the MoE block of the GPT-OSS-20B/120B-shaped programs with the experts
// split across the GPUs of one node (rank r owns experts [r*El, (r+1)*El), El = E / world).
//
// Every rank runs the same program on its own tokens (data parallel for attention, norms and the router). Per
// layer, the exchange that the reference's single-device einsums (chroma/models/gpt_oss.py:243-265,
// chroma/_src/codegen/gpu.py:390-424) never needed is done with stores into the peers' memory, so no host round
// trip or library collective sits between the routing and the expert GEMMs:
//
//   k_ep_counts       routed (token, slot) counts per global expert -> every peer's count table [src][E]; flag;
//                     wait for all tables; per owner and expert the row where this rank's rows start in the owner's
//                     grouped layout (expert-major, source-rank minor), and the local groups' row offsets
//   k_ep_dispatch     each (token, slot) claims a row and stores the token's normalised activations plus its origin
//                     (src rank, pair index) into the owning rank's receive buffer; the last CTA flags every peer
//   (local grouped SwiGLU GEMM, whose prologue waits for every rank's dispatch flag, + expert GEMM)
//   k_ep_return       each received row's expert output goes back to its source rank's return buffer at the pair
//                     index; the last CTA flags every peer
//   (k_moe_combine waits for every rank's return flag, then sums the returned rows in slot order)
//
// Synchronisation: each phase has a flag per source rank in the receiver's memory. Flags only grow: the sender
// writes the layer's epoch (a device counter every rank advances once per MoE layer, so all ranks agree) with a
// release store after a system-scope fence; the receiver polls with acquire loads. Every wait is bounded
// (EpArgs::timeout_ns of wall time): a rank that never arrives makes the waiter raise kErrTimeout and return, and
// the host reports it; the group's epochs then disagree, so it must be recreated.
// Buffer reuse across layers is safe without extra barriers: a rank can only start layer l+1's dispatch after it
// received every peer's layer-l returns, which peers send only after their layer-l GEMMs finished reading.
//
// Only plain loads and stores touch peer memory. TMA reads only this GPU's own memory (the received rows).
#pragma once

#include "tma.cuh"

namespace cb200 {

constexpr int kEpMaxWorld = 8;
constexpr int kEpMaxExperts = 256;

// Header of each rank's shared (IPC-exported) buffer.
struct EpHeader {
    unsigned cnt_flag[kEpMaxWorld];
    unsigned disp_flag[kEpMaxWorld];
    unsigned comb_flag[kEpMaxWorld];
    unsigned vrow_flag[kEpMaxWorld];  // vocab shard: final rows gathered
    unsigned vkey_flag[kEpMaxWorld];  // vocab shard: argmax keys (and logits) returned
    unsigned pad[64 - 5 * kEpMaxWorld];
    int counts[kEpMaxWorld][kEpMaxExperts];  // [src rank][global expert]
};

enum EpPhase : int { kEpCounts = 0, kEpDispatch = 1, kEpCombine = 2, kEpVocabRows = 3, kEpVocabKeys = 4 };

struct EpArgs {
    int rank, world, E, El, d;
    long long pmax;               // rows of the return buffer (pairs per rank)
    long long cap;                // rows of the receive buffer (world * pmax)
    char* peer[kEpMaxWorld];      // base of each rank's shared buffer (peer[rank] is this rank's own)
    size_t off_meta, off_x, off_y;  // offsets of the receive metadata, receive rows and return rows
    unsigned* epoch;              // this rank's epoch counter (local memory)
    unsigned* done;               // last-CTA counter (local memory)
    unsigned long long timeout_ns;  // bound of every wait for another rank
    // Vocab column shard (vrows_max == 0: off): rank r holds unembedding rows [r*Vl, r*Vl + Vr).
    int vrows_max, V, Vl;
    size_t off_vrows;             // [world * vrows_max][d] bf16: every rank's final rows
    size_t off_vkeys;             // [world][vrows_max] u64: each rank's argmax keys for this rank's rows
    size_t off_vlogits;           // [vrows_max][V] bf16: this rank's logits rows, gathered from the shards
};

__device__ __forceinline__ EpHeader* ep_header(const EpArgs& a, int r) { return reinterpret_cast<EpHeader*>(a.peer[r]); }

__device__ __forceinline__ unsigned* ep_flag(const EpArgs& a, int owner, int phase, int src) {
    EpHeader* h = ep_header(a, owner);
    switch (phase) {
        case kEpCounts: return &h->cnt_flag[src];
        case kEpDispatch: return &h->disp_flag[src];
        case kEpCombine: return &h->comb_flag[src];
        case kEpVocabRows: return &h->vrow_flag[src];
        default: return &h->vkey_flag[src];
    }
}

// Called by every thread of a CTA after its peer stores: the last CTA of the grid raises this rank's flag for
// `phase` on every peer. Classic last-block pattern at system scope: each CTA fences its stores before counting
// itself done; the last one fences again before the release stores of the flags.
__device__ __forceinline__ void ep_signal_when_last(const EpArgs& a, int phase) {
    __shared__ bool last;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(a.done, 1u);
        last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (last) {
        __threadfence_system();
        if (threadIdx.x == 0) *a.done = 0u;
        const unsigned epoch = *reinterpret_cast<volatile unsigned*>(a.epoch);
        if (threadIdx.x < unsigned(a.world)) st_release_sys(ep_flag(a, int(threadIdx.x), phase, a.rank), epoch);
    }
}

// 1 CTA. Advances the epoch, copies this rank's per-expert counts into every peer's table and flags them, clears
// the counts for the next layer, waits for every rank's counts, then plans the rows: cursor[e] = first row of this
// rank's rows for global expert e in the owner's receive buffer; offsets[0..El] = row offsets of the local experts'
// groups; *recv_total = offsets[El].
__global__ void k_ep_counts(EpArgs a, int* __restrict__ counts, int* __restrict__ cursor, int* __restrict__ offsets,
                            int* __restrict__ recv_total, unsigned* err) {
    __shared__ unsigned epoch;
    __shared__ int ok;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        epoch = *a.epoch + 1u;
        *a.epoch = epoch;
        ok = 1;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < a.world * a.E; i += blockDim.x) {
        const int q = i / a.E, e = i % a.E;
        ep_header(a, q)->counts[a.rank][e] = counts[e];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < unsigned(a.world)) st_release_sys(ep_flag(a, int(threadIdx.x), kEpCounts, a.rank), epoch);
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) counts[e] = 0;
    if (threadIdx.x < unsigned(a.world) &&
        !wait_flag_geq(&ep_header(a, a.rank)->cnt_flag[threadIdx.x], epoch, a.timeout_ns, err))
        ok = 0;
    __syncthreads();
    if (!ok) return;
    // Stage the table (written by other GPUs: volatile loads, never a stale L1 line) in shared memory, in parallel.
    __shared__ int table[kEpMaxWorld][kEpMaxExperts];
    const volatile EpHeader* h = ep_header(a, a.rank);
    for (int i = threadIdx.x; i < a.world * a.E; i += blockDim.x) table[i / a.E][i % a.E] = h->counts[i / a.E][i % a.E];
    __syncthreads();
    if (threadIdx.x < unsigned(a.world)) {  // thread q walks owner q's layout
        const int q = threadIdx.x;
        int row = 0;
        for (int el = 0; el < a.El; ++el) {
            const int e = q * a.El + el;
            if (q == a.rank) offsets[el] = row;
            for (int src = 0; src < a.world; ++src) {
                if (src == a.rank) cursor[e] = row;
                row += table[src][e];
            }
        }
        if (q == a.rank) {
            offsets[a.El] = row;
            *recv_total = row;
            if (row > a.cap) atomicOr(err, kErrIndex);
        }
    }
}

// Wait of the first `world` threads of a CTA for every rank's flag of `phase` to reach the current epoch; returns
// false (error raised) if a wait gave up. The caller synchronises the CTA afterwards.
__device__ __forceinline__ bool ep_wait_all(const EpArgs& a, int phase, unsigned* err) {
    if (threadIdx.x >= unsigned(a.world)) return true;
    const unsigned epoch = *reinterpret_cast<volatile unsigned*>(a.epoch);
    return wait_flag_geq(ep_flag(a, a.rank, phase, int(threadIdx.x)), epoch, a.timeout_ns, err);
}

// One warp per (token, slot) pair, grid-stride. Stores the token's row and its origin into the owner's buffers.
__global__ void __launch_bounds__(256) k_ep_dispatch(EpArgs a, const int* __restrict__ ridx, int pairs, int k,
                                                     const __nv_bfloat16* __restrict__ xn, int* __restrict__ cursor,
                                                     unsigned* err) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    for (int i = blockIdx.x * warps + warp; i < pairs; i += gridDim.x * warps) {
        int row = 0, q = 0;
        if (lane == 0) {
            const int e = ridx[i];
            q = e / a.El;
            row = atomicAdd(cursor + e, 1);
            if (row < a.cap)
                reinterpret_cast<int*>(a.peer[q] + a.off_meta)[row] = int(a.rank * a.pmax + i);
            else
                atomicOr(err, kErrIndex);
        }
        row = __shfl_sync(0xffffffffu, row, 0);
        q = __shfl_sync(0xffffffffu, q, 0);
        if (row >= a.cap) continue;
        const uint4* src = reinterpret_cast<const uint4*>(xn + size_t(i / k) * a.d);
        uint4* dst = reinterpret_cast<uint4*>(a.peer[q] + a.off_x) + size_t(row) * (a.d / 8);
        for (int c = lane; c < a.d / 8; c += 32) dst[c] = src[c];
    }
    ep_signal_when_last(a, kEpDispatch);
}

// One warp per received row, grid-stride: the expert output row goes back to its source rank's return buffer.
__global__ void __launch_bounds__(256) k_ep_return(EpArgs a, const __nv_bfloat16* __restrict__ y, const int* __restrict__ recv_total,
                                                   unsigned* err) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    const int total = *recv_total;
    const int* meta = reinterpret_cast<const int*>(a.peer[a.rank] + a.off_meta);
    for (int j = blockIdx.x * warps + warp; j < total && j < a.cap; j += gridDim.x * warps) {
        const long long m = __ldcg(meta + j);
        const int src = int(m / a.pmax);
        const long long i = m % a.pmax;
        if (src < 0 || src >= a.world) {
            if (lane == 0) atomicOr(err, kErrIndex);
            continue;
        }
        const uint4* from = reinterpret_cast<const uint4*>(y + size_t(j) * a.d);
        uint4* to = reinterpret_cast<uint4*>(a.peer[src] + a.off_y) + size_t(i) * (a.d / 8);
        for (int c = lane; c < a.d / 8; c += 32) to[c] = from[c];
    }
    ep_signal_when_last(a, kEpCombine);
}

// ---- Vocab column shard ---------------------------------------------------------------------------------------------
// The unembedding is split by vocab rows: every rank projects ALL ranks' final rows onto its shard, then each row's
// owner gets the shard's argmax key (and, when full logits are wanted, the shard's logits).
//
//   k_vocab_share_rows   this rank's `rows` final rows -> every rank's gather buffer at [rank * rows + r]; clears the
//                        local key array; the last CTA flags every rank (kEpVocabRows)
//   (GEMM over the world * rows gathered rows and the local shard; its prologue waits for kEpVocabRows; argmax keys
//    with the shard's column offset)
//   k_vocab_return       keys (and logits rows) of rank q's rows -> rank q; the last CTA flags every rank (kEpVocabKeys)
//   k_vocab_finish       waits for kEpVocabKeys; keys_out[r] = max over the shards' keys; logits rows copied out

// One warp per (destination rank, row), grid-stride.
__global__ void __launch_bounds__(256) k_vocab_share_rows(EpArgs a, const __nv_bfloat16* __restrict__ rows_in, int rows,
                                                          unsigned long long* __restrict__ keys_local) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.world * rows; i += gridDim.x * blockDim.x) keys_local[i] = 0ull;
    for (int i = blockIdx.x * warps + warp; i < a.world * rows; i += gridDim.x * warps) {
        const int q = i / rows, r = i % rows;
        const uint4* src = reinterpret_cast<const uint4*>(rows_in + size_t(r) * a.d);
        uint4* dst = reinterpret_cast<uint4*>(a.peer[q] + a.off_vrows) + (size_t(a.rank) * rows + r) * (a.d / 8);
        for (int c = lane; c < a.d / 8; c += 32) dst[c] = src[c];
    }
    ep_signal_when_last(a, kEpVocabRows);
}

// One warp per (destination rank q, row r of q), grid-stride. keys_local / logits_shard rows are [q * rows + r].
__global__ void __launch_bounds__(256) k_vocab_return(EpArgs a, const unsigned long long* __restrict__ keys_local,
                                                      const __nv_bfloat16* __restrict__ logits_shard, int Vr, int rows,
                                                      int want_logits) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    pdl_wait();
    pdl_trigger();
    for (int i = blockIdx.x * warps + warp; i < a.world * rows; i += gridDim.x * warps) {
        const int q = i / rows, r = i % rows;
        if (lane == 0)
            reinterpret_cast<unsigned long long*>(a.peer[q] + a.off_vkeys)[size_t(a.rank) * a.vrows_max + r] = keys_local[i];
        if (want_logits) {
            const __nv_bfloat16* src = logits_shard + size_t(i) * Vr;
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.peer[q] + a.off_vlogits) + size_t(r) * a.V +
                                 size_t(a.rank) * a.Vl;
            for (int c = lane; c < Vr; c += 32) dst[c] = src[c];
        }
    }
    ep_signal_when_last(a, kEpVocabKeys);
}

// grid-stride over rows (keys) and logits elements; every CTA first waits for all ranks' returns.
__global__ void __launch_bounds__(256) k_vocab_finish(EpArgs a, int rows, unsigned long long* __restrict__ keys_out,
                                                      __nv_bfloat16* __restrict__ logits_out, int want_logits,
                                                      unsigned* err) {
    __shared__ int ok;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if (threadIdx.x < unsigned(a.world)) {
        const unsigned epoch = *reinterpret_cast<volatile unsigned*>(a.epoch);
        if (!wait_flag_geq(ep_flag(a, a.rank, kEpVocabKeys, int(threadIdx.x)), epoch, a.timeout_ns, err)) ok = 0;
    }
    __syncthreads();
    if (!ok) return;
    const unsigned long long* table = reinterpret_cast<const unsigned long long*>(a.peer[a.rank] + a.off_vkeys);
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
        unsigned long long best = 0ull;
        for (int q = 0; q < a.world; ++q) best = max(best, __ldcg(table + size_t(q) * a.vrows_max + r));
        if (keys_out) keys_out[r] = best;
    }
    if (!want_logits) return;
    const uint4* src = reinterpret_cast<const uint4*>(a.peer[a.rank] + a.off_vlogits);
    uint4* dst = reinterpret_cast<uint4*>(logits_out);
    const size_t n16 = size_t(rows) * a.V / 8;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n16; i += size_t(gridDim.x) * blockDim.x)
        dst[i] = __ldcg(src + i);
}

}  // namespace cb200
