// One-token decode step of a dev-sized GPT-OSS model (fp32 storage) through EVERY layer in one launch: a cluster
// of kDcC CTAs on kDcC SMs exchanging activations through distributed shared memory. It replaces the per-layer
// chain k_attn_in -> k_attention -> k_out -> k_moe_up -> k_moe_down (5 dependent launches per layer, each a few
// microseconds of launch and drain latency around well under a microsecond of work) for the batch-1 decode program
// (chroma/models/cached.py:16-51 per step; the block of gpt_oss.py:189-265).
//
// Every CTA keeps its own copy of the small activations (residual x, x2, the QKV row, the attention partials, the
// expert activations) in shared memory. A phase's outputs are split over the cluster's kDcC*kWarps warps and each
// result is pushed into all kDcC copies with st.async, whose bytes complete a transaction count on the receiving
// CTA's mbarrier for that buffer; a CTA starts the next phase when its mbarrier has seen every byte. No fence or
// cluster barrier sits between phases, so weight loads issued ahead stay in flight across them.
//
//   P1  RMSNorm (per warp) -> QKV rows (2 per warp) -> +bias                     -> raw[]
//       RoPE on the gathered row (per CTA, cos/sin of the step's position computed once); CTA 0 stages the new
//       K/V rows for the commit kernel (device-resident steps: writes them into the ring slot as well)
//   P2  attention over this CTA's ceil((ctx+1)/kDcC) keys (the K/V slices of every layer are copied into shared
//       memory by cp.async at the start; the CTA holding the new token's key appends its row after RoPE), one warp
//       per query head: (max, sum, P.V) partials -> parts[]
//       every CTA merges the kDcC partials of every head with the sink logit (split-KV softmax, cached.py:36-47)
//   P3  out-projection row (1 per warp) + bias + residual                       -> x2[]
//   P4  RMSNorm + gate rows (per CTA), top-k + softmax (per warp), then one (glu, linear) row pair of each selected
//       expert per warp -> clamped SwiGLU                                        -> act[]
//   P5  mlp2 column (1 per warp) of each selected expert + bias, weighted combine in slot order + residual -> x[]
//
// The routed expert rows are known only in P4; each warp loads its rows of the 4 selected experts into registers
// right after the routing (bulk-copying every expert's rows into shared memory behind P1-P3 instead was measured
// slower: 145 KB per CTA per layer crowd the SM's inbound path and delay the exchanges).
//
// Buffer reuse is safe without barriers: a CTA reads each exchanged buffer only before it pushes its next phase's
// outputs, and a sender can only reach the same phase of the next layer after receiving those outputs.
//
// The static QKV / out / norm rows of layer l+1 are loaded into registers after P3 of layer l, its gate rows after
// P4. Each layer's weights are pulled into L2 (bulk prefetch, 1/kDcC per CTA) one layer ahead, so the L2 holds only
// the layers in flight and the vocab matrix (prefetched beside the kernel for the vocab GEMV) stays resident.
// The rounding points and summation orders of the projections are those of the per-layer kernels (gptoss.cuh);
// the attention's split over keys and its merge order differ, as in any split-KV decode.
//
// Every wait is bounded (tma.cuh's poll limit): a stuck exchange raises kErrTimeout, later waits are skipped and
// the kernel runs to its end, where one cluster barrier keeps every CTA resident until no store can target it.
#pragma once

#include "gptoss.cuh"
#include "tcgen05.cuh"

namespace cb200 {

constexpr int kDcC = 16;                 // CTAs per cluster (non-portable size: opted in at launch)
constexpr int kDcWarps = kDcC * kWarps;  // warps sharing each phase
constexpr int kDcRows1 = 2;              // QKV rows per warp
constexpr int kDcMaxK = 4;               // experts per token
constexpr int kDcMaxE = 2 * kWarps;      // gate rows (2 per warp), also <= 32 for the one-slot warp top-k

enum DcBar : int { kDcRaw = 0, kDcParts, kDcX2, kDcAct, kDcXs, kDcBars };

struct DecodeClusterArgs {
    Dims dm;
    int L, ctx, kpc;                  // layers, cache rows, keys per CTA
    const LayerW<float>* layers;      // [L]
    const int* windows;               // [L] visible-window length per layer (ctx for full-attention layers)
    const float* emb;                 // [V][d]
    const float* final_norm;          // [d]
    const float* inv_freq;            // [hd/2]
    const int64_t* tokens;            // [1]
    const int64_t* pos0;              // [1] absolute position of the new token
    const int64_t* slots;             // [ctx] absolute position held by each cache row (-1 empty)
    const float* cache_k;             // [L][ctx][KV][hd]
    const float* cache_v;
    float* new_k;                     // [L][KV][hd] staged for the commit kernel
    float* new_v;
    int* routes;                      // [L][k] or null
    const int64_t* rows;              // [1] selected row (0 or -1) or null
    float* tf;                        // [d] final-norm output for the vocab kernel
    unsigned long long* keys;         // [1] argmax key cleared for the vocab kernel, or null
    unsigned* err;
    // Device-resident decoding commits in place: the new K/V rows also go to ring slot pos0 % ctx of these caches
    // and the slot records pos0 (the commit kernel's job otherwise). Null: staging only.
    float* commit_k;
    float* commit_v;
    int64_t* commit_slots;
};

__host__ __device__ inline int dc_up4(int v) { return (v + 3) & ~3; }

// Shared-memory carve-up (in floats), identical on host and device.
struct DcLayout {
    int ps, kvs;  // floats per (CTA, head) partial; per cached key row (padded: conflict-free 16-byte reads)
    int lw, xs, raw, qkv, cs, parts, att, x2, gl, act, prow, ks, vs, total;
    __host__ __device__ DcLayout(const Dims& dm, int L, int kpc) {
        const int r1 = (dm.H + 2 * dm.KV) * dm.hd;
        ps = dc_up4(dm.hd + 2);
        kvs = dm.KV * dm.hd + 4;
        int o = 0;
        lw = o; o += dc_up4(L * int(sizeof(LayerW<float>) / 4));
        xs = o; o += dc_up4(dm.d);
        raw = o; o += dc_up4(r1);
        qkv = o; o += dc_up4(r1);
        cs = o; o += dc_up4(dm.hd);  // (cos, sin) * concentration per rotary frequency
        parts = o; o += kDcC * dm.H * ps;
        att = o; o += dc_up4(dm.H * dm.hd);
        x2 = o; o += dc_up4(dm.d);
        gl = o; o += dc_up4(dm.E);
        act = o; o += dc_up4(dm.k * dm.I);
        prow = o; o += kWarps * 32;
        ks = o; o += L * kpc * kvs;
        vs = o; o += L * kpc * kvs;
        total = o;
    }
    __host__ __device__ unsigned bytes(int bar, const Dims& dm) const {
        switch (bar) {
            case kDcRaw: return unsigned((dm.H + 2 * dm.KV) * dm.hd) * 4u;
            case kDcParts: return unsigned(kDcC * dm.H * ps) * 4u;
            case kDcX2: return unsigned(dm.d) * 4u;
            case kDcAct: return unsigned(dm.k * dm.I) * 4u;
            default: return unsigned(dm.d) * 4u;
        }
    }
};

// Remote store of 4 / 16 bytes into the shared memory of another CTA of the cluster, completing that many bytes of
// transaction on the mbarrier `bar` (a shared::cluster address in the same CTA as `addr`).
__device__ __forceinline__ void st_async_b32(uint32_t addr, float v, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr),
                 "r"(__float_as_uint(v)), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void st_async_v4(uint32_t addr, float4 v, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
                 "r"(__float_as_uint(v.x)), "r"(__float_as_uint(v.y)), "r"(__float_as_uint(v.z)),
                 "r"(__float_as_uint(v.w)), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, unsigned parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Lanes 0..kDcC-1 push `v` (uniform over the warp) to byte offset `off` of CTA `lane`'s shared memory, completing
// on that CTA's mbarrier at `bar`; `rsm` / `rbar` are the lane's shared::cluster bases of that CTA's dynamic shared
// memory and mbarrier array.
__device__ __forceinline__ void dc_push(uint32_t rsm, uint32_t rbar, uint32_t off, int bar, float v) {
    if ((threadIdx.x & 31) < kDcC) st_async_b32(rsm + off, v, rbar + 8u * unsigned(bar));
}

// Warp dot product of one weight row held as NJ float4 per lane (elements lane*4 + 128*j) with an activation row
// held the same way: per-lane FMA chain then the butterfly sum, the order of warp_gemv in gptoss.cuh.
template <int NJ>
__device__ __forceinline__ float dc_dot(const float (&w)[NJ][4], const float (&x)[NJ][4]) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        s = fmaf(w[j][0], x[j][0], s);
        s = fmaf(w[j][1], x[j][1], s);
        s = fmaf(w[j][2], x[j][2], s);
        s = fmaf(w[j][3], x[j][3], s);
    }
    return warp_sum(s);
}

template <int NJ>
__device__ __forceinline__ void dc_load(float (&w)[NJ][4], const float* row) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < NJ; ++j) load4(row + lane * 4 + 128 * j, w[j]);
}

template <int NJ>
__device__ __forceinline__ void dc_read(float (&x)[NJ][4], const float* row) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(row + lane * 4 + 128 * j);
        x[j][0] = v.x; x[j][1] = v.y; x[j][2] = v.z; x[j][3] = v.w;
    }
}

// This lane's elements of RMSNorm(x) * w, computed by every warp on its own (the reduction order of
// rows_rmsnorm: lane-strided FMA chain, butterfly sum), so no block barrier is needed.
template <int NJ>
__device__ __forceinline__ void dc_norm(float (&out)[NJ][4], const float* x, float eps, const float (&w)[NJ][4]) {
    constexpr int d = 128 * NJ;
    const int lane = threadIdx.x & 31;
    float s = 0.f;
#pragma unroll
    for (int c = lane; c < d; c += 32) s = fmaf(x[c], x[c], s);
    s = warp_sum(s);
    const float iv = 1.0f / sqrtf(s / float(d) + eps);
    dc_read<NJ>(out, x);
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) out[j][i] = __fmul_rn(__fmul_rn(out[j][i], iv), w[j][i]);
}

// Per-warp weight rows of one layer that do not depend on the routing.
template <int NJ> struct DcStatic {
    float qkv[kDcRows1][NJ][4];
    float qkv_b[kDcRows1];
    float out[NJ][4];
    float out_b;
    float gate[2][NJ][4];
    float gate_b[2];
    float attn_norm[NJ][4];
    float mlp_norm[NJ][4];
};

// The rows P1-P3 use (loaded for layer l+1 once P3 of layer l has used them) ...
template <int NJ>
__device__ __forceinline__ void dc_load_static_attn(DcStatic<NJ>& s, const LayerW<float>& w, const Dims& dm, int gw) {
    const int r1 = (dm.H + 2 * dm.KV) * dm.hd;
#pragma unroll
    for (int u = 0; u < kDcRows1; ++u) {
        const int r = gw + kDcWarps * u;
        if (r < r1) {
            dc_load<NJ>(s.qkv[u], w.qkv_w + size_t(r) * dm.d);
            s.qkv_b[u] = w.qkv_b[r];
        }
    }
    dc_load<NJ>(s.out, w.out_w + size_t(gw) * dm.H * dm.hd);
    s.out_b = w.out_b[gw];
    dc_load<NJ>(s.attn_norm, w.attn_norm);
}

// ... and the rows of P4's router (loaded for layer l+1 once P4 of layer l has computed its gate logits).
template <int NJ>
__device__ __forceinline__ void dc_load_static_mlp(DcStatic<NJ>& s, const LayerW<float>& w, const Dims& dm) {
    const int warp = threadIdx.x >> 5;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int e = warp + kWarps * u;
        if (e < dm.E) {
            dc_load<NJ>(s.gate[u], w.gate_w + size_t(e) * dm.d);
            s.gate_b[u] = w.gate_b[e];
        }
    }
    dc_load<NJ>(s.mlp_norm, w.mlp_norm);
}

// Top-k of n <= kDcMaxE gate logits in shared memory with the ranking of warp_topk_softmax (NaN highest, ties to
// the lowest index, sorted), then the softmax of the k values in slot order. Lane e holds expert e's logit as an
// orderable 64-bit key (argmax_key of the logit with -0 taken as +0) and counts the keys above its own; the lane
// of rank r owns slot r and computes its exponent and weight. Every lane ends with all k (index, weight) pairs.
__device__ __forceinline__ void dc_topk(const float* gl, int n, int k, int (&idx)[kDcMaxK], float (&wt)[kDcMaxK]) {
    const int lane = threadIdx.x & 31;
    const float g = lane < n ? gl[lane] : 0.f;
    const unsigned long long key = lane < n ? argmax_key(g + 0.0f, lane) : 0ull;
    int rank = 0;
#pragma unroll
    for (int j = 0; j < kDcMaxE; ++j) rank += __shfl_sync(0xffffffffu, key, j) > key ? 1 : 0;
    const bool sel = lane < n && rank < k;
    const float mx = warp_max(sel ? g : -INFINITY);
    const float e = sel ? expf(g - mx) : 0.f;
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < kDcMaxK; ++r) {
        const unsigned m = __ballot_sync(0xffffffffu, sel && rank == r);
        idx[r] = m ? __ffs(int(m)) - 1 : 0;
        const float er = __shfl_sync(0xffffffffu, e, idx[r]);
        if (r < k) s += er;  // slot order, as the sequential softmax
    }
    const float own = sel ? e / s : 0.f;
#pragma unroll
    for (int r = 0; r < kDcMaxK; ++r) wt[r] = r < k ? __shfl_sync(0xffffffffu, own, idx[r]) : 0.f;
}

// L2 prefetch of this CTA's 1/kDcC share of layer l's weights (its tensors are packed contiguously from attn_norm;
// the last one, b2, ends E*d floats after its start).
__device__ __forceinline__ void dc_prefetch_layer(const LayerW<float>* lws, int l, int L, const Dims& dm, int rank) {
    const char* beg = reinterpret_cast<const char*>(lws[l].attn_norm);
    const char* end = l + 1 < L ? reinterpret_cast<const char*>(lws[l + 1].attn_norm)
                                : reinterpret_cast<const char*>(lws[l].b2 + size_t(dm.E) * dm.d);
    if (end <= beg) return;  // (the host admits only layer-major packed weights)
    const size_t share = ((size_t(end - beg) + kDcC - 1) / kDcC + 15) & ~size_t(15);
    const size_t off = share * size_t(rank);
    if (off >= size_t(end - beg)) return;
    const size_t n = (size_t(end - beg) - off < share ? size_t(end - beg) - off : share) & ~size_t(15);
    for (size_t o = 0; o < n; o += 32768) bulk_prefetch_l2(beg + off + o, unsigned(n - o < 32768 ? n - o : 32768));
}

// NJ = d / 128 = H*hd / 128 = I / 128 (the host admits only d = H*hd = I = 128); HD = head_dim.
template <int NJ, int HD>
__global__ void __launch_bounds__(kThreads, 1) k_decode_cluster(DecodeClusterArgs a) {
    extern __shared__ __align__(128) float dsm[];
    __shared__ uint64_t bars[kDcBars];
    const Dims dm = a.dm;
    const DcLayout lay(dm, a.L, a.kpc);
    const LayerW<float>* lws = reinterpret_cast<const LayerW<float>*>(dsm + lay.lw);
    float* xs = dsm + lay.xs;
    float* raw = dsm + lay.raw;
    float* qkv = dsm + lay.qkv;
    float* cs = dsm + lay.cs;
    float* parts = dsm + lay.parts;
    float* att = dsm + lay.att;
    float* x2 = dsm + lay.x2;
    float* gl = dsm + lay.gl;
    float* act = dsm + lay.act;
    float* Ks = dsm + lay.ks;
    float* Vs = dsm + lay.vs;

    constexpr int d = 128 * NJ, I = 128 * NJ;
    const int rank = int(cluster_ctarank());
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = rank * kWarps + warp;
    const int H = dm.H, KV = dm.KV;
    const int r1 = (H + 2 * KV) * HD;
    const int row_kv = KV * HD, kvs = lay.kvs;
    constexpr int ps = (HD + 2 + 3) & ~3;
    const int j0 = rank * a.kpc;                         // this CTA's first key
    const int nk = max(0, min(a.kpc, a.ctx + 1 - j0));   // its keys, the new token's included
    const int nkc = max(0, min(a.kpc, a.ctx - j0));      // of which cache rows
    // shared::cluster bases of CTA `lane`'s dynamic shared memory and mbarriers (lanes < kDcC push to CTA lane).
    const uint32_t rsm = cluster_addr(dsm, uint32_t(lane % kDcC));
    const uint32_t rbar = cluster_addr(bars, uint32_t(lane % kDcC));
    auto off = [&](const float* p) { return uint32_t(p - dsm) * 4u; };
    bool live = true;  // false after a timed-out wait (thread 0)

    // Thread 0 waits (bounded) for the buffer's phase of layer l and re-arms it for layer l + 1; then the block
    // proceeds.
    auto sync = [&](int bar, int l) {
        if (threadIdx.x == 0) {
            if (live) {
                unsigned i = 0;
                while (i < kMaxPolls && !mbar_try_wait_cluster(&bars[bar], unsigned(l & 1))) ++i;
                if (i == kMaxPolls) {
                    atomicOr(a.err, kErrTimeout);
                    live = false;
                }
            }
            if (l + 1 < a.L) mbar_arrive_expect_tx(&bars[bar], lay.bytes(bar, dm));
        }
        __syncthreads();
    };

    {  // layer table -> shared memory
        const unsigned long long* src = reinterpret_cast<const unsigned long long*>(a.layers);
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(dsm + lay.lw);
        for (int i = threadIdx.x; i < a.L * int(sizeof(LayerW<float>) / 8); i += blockDim.x) dst[i] = src[i];
    }
    DcStatic<NJ> st;
    dc_load_static_attn<NJ>(st, a.layers[0], dm, gw);
    dc_load_static_mlp<NJ>(st, a.layers[0], dm);
    float fnorm[NJ][4];  // the final norm's weights, for CTA 0's last step
    dc_load<NJ>(fnorm, a.final_norm);
    if (threadIdx.x == 0) {
        for (int b = 0; b < kDcBars; ++b) mbar_init(&bars[b], 1);
        fence_barrier_init();
        for (int b = 0; b < kDcBars; ++b) mbar_arrive_expect_tx(&bars[b], lay.bytes(b, dm));
    }
    __syncthreads();
    if (threadIdx.x == 32) {  // layers 0 and 1 into L2 (later layers: one ahead, at the start of each layer)
        dc_prefetch_layer(lws, 0, a.L, dm, rank);
        if (a.L > 1) dc_prefetch_layer(lws, 1, a.L, dm, rank);
    }
    pdl_wait();
    pdl_trigger();

    // Cache slices of every layer (rows written by the previous step's commit, hence after the PDL wait).
    {
        const int row4 = row_kv / 4, per_layer = nkc * row4;
        for (int i = threadIdx.x; i < a.L * per_layer; i += blockDim.x) {
            const int l = i / per_layer, rem = i % per_layer, jj = rem / row4, c = (rem % row4) * 4;
            const size_t src = (size_t(l) * a.ctx + j0 + jj) * row_kv + c;
            const int dst = (l * a.kpc + jj) * kvs + c;
            cp_async16(Ks + dst, a.cache_k + src);
            cp_async16(Vs + dst, a.cache_v + src);
        }
        cp_async_commit();
    }
    const int64_t t_i = a.pos0[0];
    const float pos = float(t_i);  // the position k_positions would store for the single row
    const int64_t tok_row = checked_row(a.tokens[0], dm.V, false, a.err);
    // Lane jj's key of this CTA: how far before the new token it lies (the new token itself: 0) and whether its cache
    // row holds a position at all (slots -1 = empty).
    int key_age = 0;
    bool key_valid = false;
    if (lane < nk) {
        const int j = j0 + lane;
        const int64_t t_j = j < a.ctx ? a.slots[j] : t_i;
        key_valid = (j >= a.ctx || t_j >= 0) && t_j <= t_i;
        key_age = key_valid ? int(t_i - t_j < (int64_t(1) << 30) ? t_i - t_j : (int64_t(1) << 30)) : 0;
    }
    for (int j = threadIdx.x; j < HD / 2; j += blockDim.x) {
        float s, c;
        sincosf(__fmul_rn(pos, a.inv_freq[j]), &s, &c);
        cs[2 * j] = __fmul_rn(c, dm.conc);
        cs[2 * j + 1] = __fmul_rn(s, dm.conc);
    }
    for (int c = threadIdx.x; c < d; c += blockDim.x) xs[c] = a.emb[size_t(tok_row) * d + c];
    __syncthreads();
    cluster_sync_all();  // every CTA runs and has armed its mbarriers before the first remote store
    // In-place commit: every CTA has consumed its slot positions (the barrier above releases those reads), and the
    // ring slot being overwritten is masked for every reader (its old position lies ctx back, or it is empty).
    const int commit_slot = int(t_i % a.ctx);
    if (a.commit_slots && rank == 0 && threadIdx.x == 0) a.commit_slots[commit_slot] = t_i;

    // Layer l's attention sinks (lane h: head h) and window, fetched a layer ahead: read from L2 inside the
    // attention phases they sat on its critical path.
    float sink_l = lane < H ? lws[0].sinks[lane] : 0.f;
    int window_l = a.windows[0];
    for (int l = 0; l < a.L; ++l) {
        const LayerW<float>& w = lws[l];
        if (l > 0) {
            sync(kDcXs, l - 1);
            if (threadIdx.x == 32 && l + 1 < a.L) dc_prefetch_layer(lws, l + 1, a.L, dm, rank);
        }
        // ---- P1: norm, QKV rows, bias -> raw[] of every CTA
        {
            float xn[NJ][4];
            dc_norm<NJ>(xn, xs, dm.eps, st.attn_norm);
#pragma unroll
            for (int u = 0; u < kDcRows1; ++u) {
                const int r = gw + kDcWarps * u;
                if (r < r1) dc_push(rsm, rbar, off(raw + r), kDcRaw, __fadd_rn(dc_dot<NJ>(st.qkv[u], xn), st.qkv_b[u]));
            }
        }
        sync(kDcRaw, l);
        // RoPE of the q and k heads (gpt_oss.py:44-54), v heads copied; CTA 0 stages the new K/V rows.
        {
            constexpr int half = HD / 2;
            for (int i = threadIdx.x; i < (H + 2 * KV) * half; i += blockDim.x) {
                const int h = i / half, j = i % half;
                const float lo = raw[h * HD + j], hi = raw[h * HD + j + half];
                float o1 = lo, o2 = hi;
                if (h < H + KV) {
                    const float c = cs[2 * j], s = cs[2 * j + 1];
                    o1 = __fsub_rn(__fmul_rn(lo, c), __fmul_rn(hi, s));
                    o2 = __fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, s));
                }
                qkv[h * HD + j] = o1;
                qkv[h * HD + j + half] = o2;
                if (h >= H && nk > nkc) {  // the new token's K/V row is this CTA's key nkc
                    float* row = (h < H + KV ? Ks + (l * a.kpc + nkc) * kvs + (h - H) * HD
                                             : Vs + (l * a.kpc + nkc) * kvs + (h - H - KV) * HD);
                    row[j] = o1;
                    row[j + half] = o2;
                }
                if (rank == 0 && h >= H) {
                    float* dst = h < H + KV ? a.new_k + size_t(l) * row_kv + (h - H) * HD
                                            : a.new_v + size_t(l) * row_kv + (h - H - KV) * HD;
                    dst[j] = o1;
                    dst[j + half] = o2;
                    if (a.commit_k) {
                        const size_t row = (size_t(l) * a.ctx + commit_slot) * row_kv;
                        float* cdst = h < H + KV ? a.commit_k + row + (h - H) * HD : a.commit_v + row + (h - H - KV) * HD;
                        cdst[j] = o1;
                        cdst[j + half] = o2;
                    }
                }
            }
        }
        if (l == 0) cp_async_wait<0>();  // the cache slices of every layer (issued in the prologue) have landed
        __syncthreads();
        // ---- P2: attention partials over this CTA's keys, one warp per query head
        {
            const float* Kl = Ks + size_t(l) * a.kpc * kvs;
            const float* Vl = Vs + size_t(l) * a.kpc * kvs;
            const int window = window_l;
            float* prow = dsm + lay.prow + warp * 32;
            constexpr int groups = 32 / HD;
            const int g = lane / HD, dd = lane % HD;
            constexpr int chunks = ps / 4;
            for (int hq = warp; hq < H; hq += kWarps) {
                const int kvh = hq / dm.G;
                float q[HD];
#pragma unroll
                for (int e = 0; e < HD; e += 4) {
                    const float4 q4 = *reinterpret_cast<const float4*>(qkv + hq * HD + e);
                    q[e] = q4.x; q[e + 1] = q4.y; q[e + 2] = q4.z; q[e + 3] = q4.w;
                }
                float s = -INFINITY;
                if (lane < nk) {
                    const float* kr = Kl + lane * kvs + kvh * HD;
                    float kv[HD];
#pragma unroll
                    for (int e = 0; e < HD; e += 4) {
                        const float4 k4 = *reinterpret_cast<const float4*>(kr + e);
                        kv[e] = k4.x; kv[e + 1] = k4.y; kv[e + 2] = k4.z; kv[e + 3] = k4.w;
                    }
                    float dot = 0.f;
#pragma unroll
                    for (int e = 0; e < HD; ++e) dot = fmaf(q[e], kv[e], dot);
                    s = __fmul_rn(dot, dm.sm_scale);
                    if (!key_valid || (window > 0 && key_age >= window)) s = -INFINITY;
                }
                const float mx = warp_max(s);
                const float p = (lane < nk && mx != -INFINITY) ? expf(s - mx) : 0.f;
                const float lsum = warp_sum(p);
                prow[lane] = p;
                __syncwarp();
                float acc = 0.f;
#pragma unroll
                for (int i = 0; i < 32 / groups; ++i) {  // keys g, g + groups, ...
                    const int jj = g + groups * i;
                    if (jj < nk) acc = fmaf(prow[jj], Vl[jj * kvs + kvh * HD + dd], acc);
                }
#pragma unroll
                for (int o = HD; o < 32; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                // Partial = (max, sum, o[0..HD)) padded to ps floats; value i lives on lane i; pushed as float4s.
                const float ov = __shfl_sync(0xffffffffu, acc, (lane + 30) & 31);  // lane i <- o[i - 2]
                const float val = lane == 0 ? mx : (lane == 1 ? lsum : (lane < HD + 2 ? ov : 0.f));
                const uint32_t base = off(parts + (rank * H + hq) * ps);
#pragma unroll
                for (int t0 = 0; t0 < chunks * kDcC; t0 += 32) {
                    const int t = t0 + lane;
                    const int q4i = t % chunks, r = t / chunks;
                    float4 v4;
                    v4.x = __shfl_sync(0xffffffffu, val, (4 * q4i) & 31);
                    v4.y = __shfl_sync(0xffffffffu, val, (4 * q4i + 1) & 31);
                    v4.z = __shfl_sync(0xffffffffu, val, (4 * q4i + 2) & 31);
                    v4.w = __shfl_sync(0xffffffffu, val, (4 * q4i + 3) & 31);
                    const uint32_t rs = __shfl_sync(0xffffffffu, rsm, r & 31);
                    const uint32_t rb = __shfl_sync(0xffffffffu, rbar, r & 31);
                    if (t < chunks * kDcC) st_async_v4(rs + base + 16u * unsigned(q4i), v4, rb + 8u * kDcParts);
                }
                __syncwarp();
            }
        }
        sync(kDcParts, l);
        // Merge the kDcC partials of every head with its sink (the split-KV merge of k_attention), lane c holding
        // partial c's rescale factor.
        for (int hq = warp; hq < H; hq += kWarps) {
            const float sink = __shfl_sync(0xffffffffu, sink_l, hq);
            const float* ph = parts + hq * ps;
            const float mc = lane < kDcC ? ph[lane * H * ps] : -INFINITY;
            const float M = fmaxf(sink, warp_max(mc));
            const float ec = mc != -INFINITY ? expf(mc - M) : 0.f;
            const float lc = lane < kDcC ? ph[lane * H * ps + 1] : 0.f;
            const float Lsum = __fadd_rn(expf(sink - M), warp_sum(lc * ec));
            float o = 0.f;
#pragma unroll
            for (int c = 0; c < kDcC; ++c) {
                const float e = __shfl_sync(0xffffffffu, ec, c);
                if (lane < HD) o = fmaf(ph[c * H * ps + 2 + lane], e, o);
            }
            if (lane < HD) att[hq * HD + lane] = o / Lsum;
        }
        if (l + 1 < a.L) {
            sink_l = lane < H ? lws[l + 1].sinks[lane] : 0.f;
            window_l = a.windows[l + 1];
        }
        __syncthreads();
        // ---- P3: out-projection + bias + residual -> x2[]; then the next layer's P1-P3 rows
        {
            float av[NJ][4];
            dc_read<NJ>(av, att);
            dc_push(rsm, rbar, off(x2 + gw), kDcX2, __fadd_rn(xs[gw], __fadd_rn(dc_dot<NJ>(st.out, av), st.out_b)));
        }
        if (l + 1 < a.L) dc_load_static_attn<NJ>(st, lws[l + 1], dm, gw);
        sync(kDcX2, l);
        // ---- P4: norm and gate rows (per CTA), top-k and softmax (per warp), one mlp1 pair of each selected expert
        float xn[NJ][4];
        dc_norm<NJ>(xn, x2, dm.eps, st.mlp_norm);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int e = warp + kWarps * u;
            if (e < dm.E) {
                const float acc = dc_dot<NJ>(st.gate[u], xn);
                if (lane == 0) gl[e] = __fadd_rn(acc, st.gate_b[u]);
            }
        }
        if (l + 1 < a.L) dc_load_static_mlp<NJ>(st, lws[l + 1], dm);
        __syncthreads();
        int sidx[kDcMaxK];
        float sw[kDcMaxK];
        dc_topk(gl, dm.E, dm.k, sidx, sw);
        if (rank == 0 && warp == 0 && a.routes) {
#pragma unroll
            for (int r = 0; r < kDcMaxK; ++r)
                if (r == lane && r < dm.k) a.routes[size_t(l) * dm.k + r] = sidx[r];
        }
        int ex[kDcMaxK];
#pragma unroll
        for (int u = 0; u < kDcMaxK; ++u) ex[u] = u < dm.k ? int(checked_row(sidx[u], dm.E, true, a.err)) : 0;
        // Routed rows: warp gw's mlp1 pair gw and mlp2 row gw of each selected expert (+ biases).
        float wg[kDcMaxK][NJ][4], wl[kDcMaxK][NJ][4], w2r[kDcMaxK][NJ][4], bg[kDcMaxK], bl[kDcMaxK], bd[kDcMaxK];
#pragma unroll
        for (int u = 0; u < kDcMaxK; ++u) {
            if (u < dm.k) {
                const int e = ex[u];
                const float* W1 = w.w1 + (size_t(e) * 2 * I + 2 * gw) * d;
                dc_load<NJ>(wg[u], W1);
                dc_load<NJ>(wl[u], W1 + d);
                bg[u] = w.b1[size_t(e) * 2 * I + 2 * gw];
                bl[u] = w.b1[size_t(e) * 2 * I + 2 * gw + 1];
                dc_load<NJ>(w2r[u], w.w2 + (size_t(e) * d + gw) * I);
                bd[u] = w.b2[size_t(e) * d + gw];
            }
        }
#pragma unroll
        for (int u = 0; u < kDcMaxK; ++u) {
            if (u < dm.k) {
                const float hg = __fadd_rn(dc_dot<NJ>(wg[u], xn), bg[u]);
                const float hlin = __fadd_rn(dc_dot<NJ>(wl[u], xn), bl[u]);
                // Clamped SwiGLU (gpt_oss.py:212-219), the arithmetic of k_moe_up.
                const float glu = fminf(hg, dm.limit);
                const float lin = fminf(fmaxf(hlin, -dm.limit), dm.limit);
                const float z = __fmul_rn(glu, dm.alpha);
                const float sg = 1.0f / (1.0f + expf(-z));
                const float og = __fmul_rn(glu, sg);
                const float l1 = __fadd_rn(lin, 1.0f);
                dc_push(rsm, rbar, off(act + u * I + gw), kDcAct, __fmul_rn(og, l1));
            }
        }
        sync(kDcAct, l);
        // ---- P5: mlp2 columns, weighted combine in slot order, residual -> x[]
        {
            float comb = 0.f;
#pragma unroll
            for (int u = 0; u < kDcMaxK; ++u) {
                if (u < dm.k) {
                    float av[NJ][4];
                    dc_read<NJ>(av, act + u * I);
                    comb = __fadd_rn(comb, __fmul_rn(__fadd_rn(dc_dot<NJ>(w2r[u], av), bd[u]), sw[u]));
                }
            }
            dc_push(rsm, rbar, off(xs + gw), kDcXs, __fadd_rn(x2[gw], comb));
        }
    }
    sync(kDcXs, a.L - 1);

    // Final RMSNorm of the token's row (gpt_oss.py:309) for the vocab kernel; clears the argmax key.
    if (rank == 0 && warp == 0) {
        if (a.rows && lane == 0) checked_row(a.rows[0], 1, true, a.err);
        float out[NJ][4];
        dc_norm<NJ>(out, xs, dm.eps, fnorm);
#pragma unroll
        for (int j = 0; j < NJ; ++j)
            *reinterpret_cast<float4*>(a.tf + lane * 4 + 128 * j) = make_float4(out[j][0], out[j][1], out[j][2], out[j][3]);
        if (lane == 0 && a.keys) a.keys[0] = 0ull;
    }
    cluster_sync_all();  // no CTA leaves while another may still store into it
}

}  // namespace cb200
