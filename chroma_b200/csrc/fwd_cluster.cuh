// Forward pass of up to 8 tokens of a dev-sized GPT-OSS model (fp32 storage, no KV cache: the reference's 8-token
// `Program(tokens)`, chroma/models/gpt_oss.py:189-310) through EVERY layer in one launch: a cluster of kDcC CTAs
// on kDcC SMs exchanging activations through distributed shared memory, the multi-token sibling of
// k_decode_cluster. It replaces the per-layer chain k_attn_in -> k_attention -> k_out -> k_moe_up -> k_moe_down
// (5 dependent launches per layer, a few microseconds each around well under a microsecond of work).
//
// Every CTA keeps all n token rows of the small activations in shared memory. Each phase's outputs are split over
// the cluster's 128 warps and pushed into all kDcC copies with st.async, completing a transaction count on the
// receiving CTA's mbarrier for that buffer (as in k_decode_cluster):
//
//   P1  RMSNorm of the n rows (per warp) -> QKV rows gw, gw + 128 for every token -> +bias         -> raw[t][r]
//       RoPE of every token's q and k heads (per CTA)                                             -> qkv[t][r]
//   P2  one warp per (query row, head) pair: scores over the causal keys, sink, softmax, P.V      -> att[t][h*hd]
//   P3  out-projection row gw for every token + bias + residual                                   -> x2[t][c]
//   P4  RMSNorm + gate rows + top-k + softmax of every token (per CTA); then the (glu, linear) pair gw of every
//       expert some token selected, SwiGLU for the (token, slot) pairs routed to it                -> act[t][s][i]
//   P5  mlp2 column gw of each (token, slot) pair's expert + bias, weighted combine in slot order + residual
//                                                                                                  -> xs[t][c]
//
// A weight row is held once in registers and dotted with all n tokens; the n per-lane partial sums are reduced
// with a reduce-scatter (rs8 / rs32) whose pairing of lanes, level by level, is warp_sum's butterfly, so every
// token's sum goes through the same additions in the same tree as the per-layer kernels' warp_sum: the projections,
// norms, attention, routing and combine are bit-identical to the per-layer chain (gptoss.cuh), the final norm to
// k_final_norm's. After rs8 lane L holds token L >> 2's sum; after rs32, pair L's.
//
// Buffer reuse needs no barrier for the reason given in decode_cluster.cuh: a CTA reads each exchanged buffer only
// before it pushes its next phase's outputs, and a sender reaches the same phase of the next layer only after
// receiving those outputs. Every wait is bounded (tma.cuh's poll limit); a stuck exchange raises kErrTimeout, later
// waits are skipped, and one cluster barrier at the end keeps every CTA resident until no store can target it.
#pragma once

#include "decode_cluster.cuh"

namespace cb200 {

constexpr int kFcTok = 8;   // tokens per launch (at most)

enum FcBar : int { kFcRaw = 0, kFcAtt, kFcX2, kFcAct, kFcXs, kFcBars };

struct FwdClusterArgs {
    Dims dm;
    int L, n;
    const LayerW<float>* layers;  // [L]
    const int* windows;           // [L] causal window per layer (0: none)
    const float* emb;             // [V][d]
    const float* final_norm;      // [d]
    const float* inv_freq;        // [hd/2]
    const float* positions;       // [n]
    const int64_t* tokens;        // [n]
    const int64_t* rows;          // [1] the row whose logits are wanted (last-row programs), or null: every row
    int* routes;                  // [L][n][k] or null
    float* tf;                    // [rows][d] final-norm rows for the vocab kernel
    unsigned long long* keys;     // argmax keys cleared for the vocab kernel, or null
    unsigned* err;
};

// Shared-memory carve-up (floats), identical on host and device.
struct FcLayout {
    int lw, xs, raw, qkv, cs, att, x2, gl, sw, act, sidx, stg, w1s, w2s, total;
    __host__ __device__ FcLayout(const Dims& dm, int L) {
        const int r1 = (dm.H + 2 * dm.KV) * dm.hd;
        int o = 0;
        lw = o; o += dc_up4(L * int(sizeof(LayerW<float>) / 4));
        xs = o; o += kFcTok * dm.d;
        raw = o; o += kFcTok * dc_up4(r1);
        qkv = o; o += kFcTok * dc_up4(r1);
        cs = o; o += kFcTok * dc_up4(dm.hd);
        att = o; o += kFcTok * dm.H * dm.hd;
        x2 = o; o += kFcTok * dm.d;
        gl = o; o += kFcTok * dc_up4(dm.E);
        sw = o; o += kFcTok * kDcMaxK;
        act = o; o += kFcTok * kDcMaxK * dm.I;
        sidx = o; o += kFcTok * kDcMaxK;  // ints
        stg = o; o += kFcTok * kDcMaxK * kWarps;  // this CTA's results of a phase, before they are pushed
        w1s = o; o += kWarps * dm.E * 2 * dm.I;  // per warp: its (glu, linear) pair of every expert
        w2s = o; o += kWarps * dm.E * dm.d;      // per warp: its mlp2 row of every expert
        total = o;
    }
    __host__ __device__ unsigned bytes(int bar, const Dims& dm, int n) const {
        switch (bar) {
            case kFcRaw: return unsigned(n * (dm.H + 2 * dm.KV) * dm.hd) * 4u;
            case kFcAtt: return unsigned(n * dm.H * dm.hd) * 4u;
            case kFcAct: return unsigned(n * dm.k * dm.I) * 4u;
            default: return unsigned(n * dm.d) * 4u;  // x2, xs
        }
    }
};

// Reduce-scatter of 8 per-lane partial sums: lane L returns the warp-wide sum of v[L >> 2], through the pairings
// of warp_sum (xor 16, 8, 4, then 2, 1), each addition own + partner as there.
__device__ __forceinline__ float rs8(const float (&v)[8]) {
    const int lane = threadIdx.x & 31;
    float u[4], w[2];
    {
        const bool hi = lane & 16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float keep = hi ? v[i + 4] : v[i], send = hi ? v[i] : v[i + 4];
            u[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
        }
    }
    {
        const bool hi = lane & 8;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const float keep = hi ? u[i + 2] : u[i], send = hi ? u[i] : u[i + 2];
            w[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
        }
    }
    const bool hi = lane & 4;
    float x = (hi ? w[1] : w[0]) + __shfl_xor_sync(0xffffffffu, hi ? w[0] : w[1], 4);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    return x;
}

// Reduce-scatter of 32 per-lane partial sums: lane L returns the warp-wide sum of v[L] (warp_sum's pairings).
__device__ __forceinline__ float rs32(const float (&v)[32]) {
    const int lane = threadIdx.x & 31;
    float a[16], b[8], c[4], d2[2];
    {
        const bool hi = lane & 16;
#pragma unroll
        for (int i = 0; i < 16; ++i) a[i] = (hi ? v[i + 16] : v[i]) + __shfl_xor_sync(0xffffffffu, hi ? v[i] : v[i + 16], 16);
    }
    {
        const bool hi = lane & 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) b[i] = (hi ? a[i + 8] : a[i]) + __shfl_xor_sync(0xffffffffu, hi ? a[i] : a[i + 8], 8);
    }
    {
        const bool hi = lane & 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i] = (hi ? b[i + 4] : b[i]) + __shfl_xor_sync(0xffffffffu, hi ? b[i] : b[i + 4], 4);
    }
    {
        const bool hi = lane & 2;
#pragma unroll
        for (int i = 0; i < 2; ++i) d2[i] = (hi ? c[i + 2] : c[i]) + __shfl_xor_sync(0xffffffffu, hi ? c[i] : c[i + 2], 2);
    }
    const bool hi = lane & 1;
    return (hi ? d2[1] : d2[0]) + __shfl_xor_sync(0xffffffffu, hi ? d2[0] : d2[1], 1);
}

// Per-lane partial of row . x over this lane's 4 elements (lane*4 .. lane*4 + 3, d = 128): warp_gemv's FMA chain.
__device__ __forceinline__ float fc_part(const float (&w)[1][4], const float (&x)[4]) {
    float s = fmaf(w[0][0], x[0], 0.f);
    s = fmaf(w[0][1], x[1], s);
    s = fmaf(w[0][2], x[2], s);
    return fmaf(w[0][3], x[3], s);
}

// This lane's 4 elements of RMSNorm(x_t) * w for every token t < n (rows_rmsnorm's order: lane-strided FMA chain,
// butterfly sum, here reduce-scattered and the n inverse norms shared back from lanes 4t).
__device__ __forceinline__ void fc_norm(float (&out)[kFcTok][4], const float* x, int n, float eps,
                                        const float (&w)[1][4]) {
    const int lane = threadIdx.x & 31;
    float s[kFcTok];
#pragma unroll
    for (int t = 0; t < kFcTok; ++t) {
        s[t] = 0.f;
        if (t < n)
#pragma unroll
            for (int c = lane; c < 128; c += 32) s[t] = fmaf(x[t * 128 + c], x[t * 128 + c], s[t]);
    }
    const float tot = rs8(s);
    const float iv_own = 1.0f / sqrtf(tot / 128.f + eps);
#pragma unroll
    for (int t = 0; t < kFcTok; ++t) {
        const float iv = __shfl_sync(0xffffffffu, iv_own, 4 * t);
        if (t < n) {
            const float4 v = *reinterpret_cast<const float4*>(x + t * 128 + lane * 4);
            out[t][0] = __fmul_rn(__fmul_rn(v.x, iv), w[0][0]);
            out[t][1] = __fmul_rn(__fmul_rn(v.y, iv), w[0][1]);
            out[t][2] = __fmul_rn(__fmul_rn(v.z, iv), w[0][2]);
            out[t][3] = __fmul_rn(__fmul_rn(v.w, iv), w[0][3]);
        } else {
            out[t][0] = out[t][1] = out[t][2] = out[t][3] = 0.f;
        }
    }
}

// One weight row (in registers) dotted with every token's row: lane L returns token L >> 2's sum.
__device__ __forceinline__ float fc_dot8(const float (&w)[1][4], const float (&x)[kFcTok][4]) {
    float v[kFcTok];
#pragma unroll
    for (int t = 0; t < kFcTok; ++t) v[t] = fc_part(w, x[t]);
    return rs8(v);
}

// NJ = 1 and d = H*hd = I = 128 (the host admits only those widths); HD = head_dim.
template <int HD>
__global__ void __launch_bounds__(kThreads, 1) k_fwd_cluster(FwdClusterArgs a) {
    extern __shared__ __align__(128) float fsm[];
    __shared__ uint64_t bars[kFcBars];
    __shared__ uint32_t rsm_tab[kDcC], rbar_tab[kDcC];
    __shared__ unsigned chosen_experts;  // union of the layer's routed experts (bit e)
    const Dims dm = a.dm;
    const FcLayout lay(dm, a.L);
    const LayerW<float>* lws = reinterpret_cast<const LayerW<float>*>(fsm + lay.lw);
    float* xs = fsm + lay.xs;
    float* raw = fsm + lay.raw;
    float* qkv = fsm + lay.qkv;
    float* cs = fsm + lay.cs;
    float* att = fsm + lay.att;
    float* x2 = fsm + lay.x2;
    float* gl = fsm + lay.gl;
    float* swv = fsm + lay.sw;
    float* act = fsm + lay.act;
    int* sidx = reinterpret_cast<int*>(fsm + lay.sidx);
    float* stg = fsm + lay.stg;
    float* w1s = fsm + lay.w1s + size_t(threadIdx.x >> 5) * dm.E * 2 * 128;  // this warp's [E][2][128]
    float* w2s = fsm + lay.w2s + size_t(threadIdx.x >> 5) * dm.E * 128;      // this warp's [E][128]

    constexpr int d = 128, I = 128, half = HD / 2;
    const int n = a.n;
    const int rank = int(cluster_ctarank());
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = rank * kWarps + warp;
    const int H = dm.H, KV = dm.KV, G = dm.G, E = dm.E, k = dm.k;
    const int r1 = (H + 2 * KV) * HD, r1p = dc_up4(r1), hdp = dc_up4(HD), ep = dc_up4(E);
    const int tj = lane >> 2, tm = lane & 3;  // after rs8: this lane's token; its share of the 16 CTAs
    auto off = [&](const float* p) { return uint32_t(p - fsm) * 4u; };
    // The CTA's threads push `chunks` 16-byte chunks (source src(c), destination dst(c)) into every CTA.
    auto push_chunks = [&](int chunks, auto src, auto dst, int bar) {
        for (int it = threadIdx.x; it < chunks * kDcC; it += blockDim.x) {
            const int cta = it % kDcC, c = it / kDcC;
            st_async_v4(rsm_tab[cta] + off(dst(c)), *reinterpret_cast<const float4*>(src(c)),
                        rbar_tab[cta] + 8u * unsigned(bar));
        }
    };
    bool live = true;  // false after a timed-out wait (thread 0)
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
            if (l + 1 < a.L) mbar_arrive_expect_tx(&bars[bar], lay.bytes(bar, dm, n));
        }
        __syncthreads();
    };

    {  // layer table -> shared memory
        const unsigned long long* src = reinterpret_cast<const unsigned long long*>(a.layers);
        unsigned long long* dst = reinterpret_cast<unsigned long long*>(fsm + lay.lw);
        for (int i = threadIdx.x; i < a.L * int(sizeof(LayerW<float>) / 8); i += blockDim.x) dst[i] = src[i];
    }
    if (threadIdx.x < kDcC) {
        rsm_tab[threadIdx.x] = cluster_addr(fsm, threadIdx.x);
        rbar_tab[threadIdx.x] = cluster_addr(bars, threadIdx.x);
    }
    DcStatic<1> st;
    dc_load_static_attn<1>(st, a.layers[0], dm, gw);
    dc_load_static_mlp<1>(st, a.layers[0], dm);
    float fnorm[1][4];
    dc_load<1>(fnorm, a.final_norm);
    if (threadIdx.x == 0) {
        for (int b = 0; b < kFcBars; ++b) mbar_init(&bars[b], 1);
        fence_barrier_init();
        for (int b = 0; b < kFcBars; ++b) mbar_arrive_expect_tx(&bars[b], lay.bytes(b, dm, n));
    }
    __syncthreads();
    if (threadIdx.x == 32) {  // layers 0 and 1 into L2 (later layers: one ahead, at the start of each layer)
        dc_prefetch_layer(lws, 0, a.L, dm, rank);
        if (a.L > 1) dc_prefetch_layer(lws, 1, a.L, dm, rank);
    }
    pdl_wait();
    pdl_trigger();
    // Embedding rows (bounds-checked ids), the rotary (cos, sin) * concentration of every token's position; rows
    // past n are zero.
    __shared__ int64_t tok_row[kFcTok];
    if (threadIdx.x < unsigned(n)) tok_row[threadIdx.x] = checked_row(a.tokens[threadIdx.x], dm.V, false, a.err);
    __syncthreads();
    for (int i = threadIdx.x; i < kFcTok * d; i += blockDim.x) {
        const int t = i / d, c = i % d;
        xs[i] = t < n ? a.emb[size_t(tok_row[t]) * d + c] : 0.f;
        att[i] = 0.f;
    }
    for (int i = threadIdx.x; i < n * half; i += blockDim.x) {
        const int t = i / half, j = i % half;
        float s, c;
        sincosf(__fmul_rn(a.positions[t], a.inv_freq[j]), &s, &c);
        cs[t * hdp + 2 * j] = __fmul_rn(c, dm.conc);
        cs[t * hdp + 2 * j + 1] = __fmul_rn(s, dm.conc);
    }
    // This warp's expert rows of layer l (P4's mlp1 pair gw and P5's mlp2 row gw of every expert) into shared
    // memory and its biases onto lanes e < E, issued a whole layer ahead (after P5 of layer l - 1): whichever
    // experts the routing picks, P4 and P5 then read nothing from L2.
    float bg_l = 0.f, bl_l = 0.f, bd_l = 0.f, sink_l = 0.f;  // lane e: expert e's biases; lane h: head h's sink
    int window_l = 0;
    auto stage_experts = [&](int l) {
        const LayerW<float>& w = lws[l];
        if (lane < H) sink_l = w.sinks[lane];
        window_l = a.windows[l];
        for (int e = 0; e < E; ++e) {
            const float* W1 = w.w1 + (size_t(e) * 2 * I + 2 * gw) * d + lane * 4;
            cp_async16(w1s + (2 * e) * 128 + lane * 4, W1);
            cp_async16(w1s + (2 * e + 1) * 128 + lane * 4, W1 + d);
            cp_async16(w2s + e * 128 + lane * 4, w.w2 + (size_t(e) * d + gw) * I + lane * 4);
        }
        cp_async_commit();
        if (lane < E) {
            bg_l = w.b1[size_t(lane) * 2 * I + 2 * gw];
            bl_l = w.b1[size_t(lane) * 2 * I + 2 * gw + 1];
            bd_l = w.b2[size_t(lane) * d + gw];
        }
    };
    stage_experts(0);
    __syncthreads();
    cluster_sync_all();  // every CTA runs and has armed its mbarriers before the first remote store

    for (int l = 0; l < a.L; ++l) {
        if (l > 0) {
            sync(kFcXs, l - 1);
            if (threadIdx.x == 32 && l + 1 < a.L) dc_prefetch_layer(lws, l + 1, a.L, dm, rank);
        }
        // ---- P1: norm, QKV rows gw and gw + 128 of every token, bias -> raw[] of every CTA
        {
            float xn[kFcTok][4];
            fc_norm(xn, xs, n, dm.eps, st.attn_norm);
#pragma unroll
            for (int u = 0; u < kDcRows1; ++u) {
                const int r = gw + kDcWarps * u;
                if (r < r1) {
                    const float v = __fadd_rn(fc_dot8(st.qkv[u], xn), st.qkv_b[u]);
                    if (tj < n && tm == 0) stg[(tj * 2 + u) * kWarps + warp] = v;
                }
            }
        }
        __syncthreads();
        // Rows 128u + 8 rank .. + 7 of token t (r1 is a multiple of 8: a block is whole or absent).
        {
            const int ublocks = rank * kWarps + kDcWarps < r1 ? 2 : 1;
            push_chunks(
                n * ublocks * 2, [&](int c) { return stg + ((c / (2 * ublocks)) * 2 + (c / 2) % ublocks) * kWarps + 4 * (c % 2); },
                [&](int c) { return raw + (c / (2 * ublocks)) * r1p + kDcWarps * ((c / 2) % ublocks) + rank * kWarps + 4 * (c % 2); },
                kFcRaw);
        }
        sync(kFcRaw, l);
        // RoPE of every token's q and k heads (k_attn_in's arithmetic), v heads copied.
        for (int i = threadIdx.x; i < n * (H + 2 * KV) * half; i += blockDim.x) {
            const int t = i / ((H + 2 * KV) * half), rem = i % ((H + 2 * KV) * half);
            const int h = rem / half, j = rem % half;
            const float lo = raw[t * r1p + h * HD + j], hi = raw[t * r1p + h * HD + j + half];
            float o1 = lo, o2 = hi;
            if (h < H + KV) {
                const float c = cs[t * hdp + 2 * j], s = cs[t * hdp + 2 * j + 1];
                o1 = __fsub_rn(__fmul_rn(lo, c), __fmul_rn(hi, s));
                o2 = __fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, s));
            }
            qkv[t * r1p + h * HD + j] = o1;
            qkv[t * r1p + h * HD + j + half] = o2;
        }
        __syncthreads();
        // ---- P2: one warp per (query row, head): k_attention's single-chunk arithmetic, key jj on lane jj
        if (gw < n * H) {
            const int i = gw / H, hq = gw % H, kvh = hq / G;
            const int window = window_l;
            const float* qr = qkv + i * r1p + hq * HD;
            float s = -INFINITY;
            if (lane < n) {
                const float* kr = qkv + lane * r1p + (H + kvh) * HD;
                float qv[HD], kv[HD];  // both rows loaded before the FMA chain
#pragma unroll
                for (int e = 0; e < HD; e += 4) {
                    const float4 q4 = *reinterpret_cast<const float4*>(qr + e);
                    const float4 k4 = *reinterpret_cast<const float4*>(kr + e);
                    qv[e] = q4.x; qv[e + 1] = q4.y; qv[e + 2] = q4.z; qv[e + 3] = q4.w;
                    kv[e] = k4.x; kv[e + 1] = k4.y; kv[e + 2] = k4.z; kv[e + 3] = k4.w;
                }
                float dot = 0.f;
#pragma unroll
                for (int e = 0; e < HD; ++e) dot = fmaf(qv[e], kv[e], dot);
                s = __fmul_rn(dot, dm.sm_scale);
                if (!(lane <= i && (window <= 0 || i - lane < window))) s = -INFINITY;
            }
            const float mx = warp_max(s);
            const float sink = __shfl_sync(0xffffffffu, sink_l, hq);
            const float ref = fmaxf(mx, sink);
            float p = (lane < n && ref != -INFINITY) ? expf(s - ref) : 0.f;
            float lsum = warp_sum(p);
            lsum += expf(sink - ref);
            p = p / lsum;
            constexpr int groups = 32 / HD;
            const int g = lane / HD, dd = lane % HD;
            float acc = 0.f;
#pragma unroll
            for (int it = 0; it < (kFcTok + groups - 1) / groups; ++it) {
                const int jj = g + groups * it;
                const float pj = __shfl_sync(0xffffffffu, p, jj < 32 ? jj : 31);
                if (jj < n) acc = fmaf(pj, qkv[jj * r1p + (H + KV + kvh) * HD + dd], acc);
            }
#pragma unroll
            for (int o = HD; o < 32; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            // o[dd] is on lanes dd, dd + HD, ...: the HD / 4 chunks x 16 CTAs go out as 16-byte stores.
            constexpr int nq = HD / 4, per_lane = nq * kDcC / 32;
            const int qc = lane % nq;
            float4 o4;
            o4.x = __shfl_sync(0xffffffffu, acc, 4 * qc);
            o4.y = __shfl_sync(0xffffffffu, acc, 4 * qc + 1);
            o4.z = __shfl_sync(0xffffffffu, acc, 4 * qc + 2);
            o4.w = __shfl_sync(0xffffffffu, acc, 4 * qc + 3);
#pragma unroll
            for (int q = 0; q < per_lane; ++q) {
                const int cta = lane / nq + (32 / nq) * q;
                st_async_v4(rsm_tab[cta] + off(att + i * H * HD + hq * HD + 4 * qc), o4, rbar_tab[cta] + 8u * kFcAtt);
            }
        }
        sync(kFcAtt, l);
        // ---- P3: out-projection row gw of every token + bias + residual -> x2[]; then the next layer's P1-P3 rows
        {
            float av[kFcTok][4];
#pragma unroll
            for (int t = 0; t < kFcTok; ++t) {
                const float4 v = *reinterpret_cast<const float4*>(att + t * d + lane * 4);
                av[t][0] = v.x; av[t][1] = v.y; av[t][2] = v.z; av[t][3] = v.w;
            }
            const float v = fc_dot8(st.out, av);
            if (tj < n && tm == 0) stg[tj * kWarps + warp] = __fadd_rn(xs[tj * d + gw], __fadd_rn(v, st.out_b));
        }
        __syncthreads();
        push_chunks(2 * n, [&](int c) { return stg + (c / 2) * kWarps + 4 * (c % 2); },
                    [&](int c) { return x2 + (c / 2) * d + rank * kWarps + 4 * (c % 2); }, kFcX2);
        if (l + 1 < a.L) dc_load_static_attn<1>(st, lws[l + 1], dm, gw);
        sync(kFcX2, l);
        // ---- P4: norm and gate rows of every token (per CTA), top-k and softmax (warp t: token t)
        float xn[kFcTok][4];
        fc_norm(xn, x2, n, dm.eps, st.mlp_norm);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int e = warp + kWarps * u;
            if (e < E) {
                const float v = fc_dot8(st.gate[u], xn);
                if (tm == 0 && tj < n) gl[tj * ep + e] = __fadd_rn(v, st.gate_b[u]);
            }
        }
        if (l + 1 < a.L) dc_load_static_mlp<1>(st, lws[l + 1], dm);
        if (threadIdx.x == 0) chosen_experts = 0u;
        __syncthreads();
        if (warp < n) {
            int idx[kDcMaxK];
            float wt[kDcMaxK];
            dc_topk(gl + warp * ep, E, k, idx, wt);
#pragma unroll
            for (int r = 0; r < kDcMaxK; ++r) {
                if (lane == r && r < k) {
                    sidx[warp * kDcMaxK + r] = idx[r];
                    swv[warp * kDcMaxK + r] = wt[r];
                    atomicOr(&chosen_experts, 1u << idx[r]);
                    if (rank == 0 && a.routes) a.routes[(size_t(l) * n + warp) * k + r] = idx[r];
                }
            }
        }
        __syncthreads();
        // The (glu, linear) pair gw of every expert some token selected; lane 4t + s keeps (token t, slot s)'s
        // SwiGLU output (k_moe_up's arithmetic).
        {
            const unsigned chosen = chosen_experts;
            const int my_e = (tj < n && tm < k) ? sidx[tj * kDcMaxK + tm] : -1;
            float my_act = 0.f;
            cp_async_wait<0>();
            __syncwarp();
            // Three experts per pass, so their reduction chains overlap.
            auto swiglu = [&](int e, float ag, float al) {
                const float bg = __shfl_sync(0xffffffffu, bg_l, e), bl = __shfl_sync(0xffffffffu, bl_l, e);
                if (my_e == e) {
                    const float hg = __fadd_rn(ag, bg);
                    const float hl = __fadd_rn(al, bl);
                    const float glu = fminf(hg, dm.limit);
                    const float lin = fminf(fmaxf(hl, -dm.limit), dm.limit);
                    const float z = __fmul_rn(glu, dm.alpha);
                    const float sg = 1.0f / (1.0f + expf(-z));
                    const float og = __fmul_rn(glu, sg);
                    my_act = __fmul_rn(og, __fadd_rn(lin, 1.0f));
                }
            };
            for (unsigned um = chosen; um;) {
                const int e0 = __ffs(int(um)) - 1;
                um &= um - 1;
                const int e1 = um ? __ffs(int(um)) - 1 : e0;
                if (um) um &= um - 1;
                const int e2 = um ? __ffs(int(um)) - 1 : e0;
                if (um) um &= um - 1;
                float wg0[1][4], wl0[1][4], wg1[1][4], wl1[1][4], wg2[1][4], wl2[1][4];
                dc_read<1>(wg0, w1s + (2 * e0) * 128);
                dc_read<1>(wl0, w1s + (2 * e0 + 1) * 128);
                dc_read<1>(wg1, w1s + (2 * e1) * 128);
                dc_read<1>(wl1, w1s + (2 * e1 + 1) * 128);
                dc_read<1>(wg2, w1s + (2 * e2) * 128);
                dc_read<1>(wl2, w1s + (2 * e2 + 1) * 128);
                const float ag0 = fc_dot8(wg0, xn), al0 = fc_dot8(wl0, xn);
                const float ag1 = fc_dot8(wg1, xn), al1 = fc_dot8(wl1, xn);
                const float ag2 = fc_dot8(wg2, xn), al2 = fc_dot8(wl2, xn);
                swiglu(e0, ag0, al0);
                if (e1 != e0) swiglu(e1, ag1, al1);
                if (e2 != e0) swiglu(e2, ag2, al2);
            }
            if (my_e >= 0) stg[(tj * kDcMaxK + tm) * kWarps + warp] = my_act;
        }
        __syncthreads();
        // (token t, slot s < k) chunk pairs: act[t][s][8 rank .. + 7].
        push_chunks(2 * n * k,
                    [&](int c) { return stg + ((c / (2 * k)) * kDcMaxK + (c / 2) % k) * kWarps + 4 * (c % 2); },
                    [&](int c) { return act + ((c / (2 * k)) * kDcMaxK + (c / 2) % k) * I + rank * kWarps + 4 * (c % 2); },
                    kFcAct);
        sync(kFcAct, l);
        // ---- P5: mlp2 column gw of every (token, slot) pair's expert + bias, weighted combine in slot order
        // (k_moe_down's arithmetic), residual -> xs[] of every CTA
        {
            float v[kFcTok * kDcMaxK];
#pragma unroll
            for (int p = 0; p < kFcTok * kDcMaxK; ++p) {
                const int t = p / kDcMaxK, s = p % kDcMaxK;
                v[p] = 0.f;
                if (t < n && s < k) {
                    float w2r[1][4];
                    dc_read<1>(w2r, w2s + sidx[p] * 128);
                    const float4 av = *reinterpret_cast<const float4*>(act + p * I + lane * 4);
                    float s4 = fmaf(w2r[0][0], av.x, 0.f);
                    s4 = fmaf(w2r[0][1], av.y, s4);
                    s4 = fmaf(w2r[0][2], av.z, s4);
                    v[p] = fmaf(w2r[0][3], av.w, s4);
                }
            }
            const float part = rs32(v);  // pair `lane`
            const float bd = __shfl_sync(0xffffffffu, bd_l, (tj < n && tm < k) ? sidx[lane] : 0);
            float term = 0.f;
            if (tj < n && tm < k) {
                const float y = __fadd_rn(part, bd);
                term = __fmul_rn(y, swv[lane]);
            }
            float comb = 0.f;
            for (int u = 0; u < k; ++u) comb = __fadd_rn(comb, __shfl_sync(0xffffffffu, term, (lane & ~3) + u));
            if (tj < n && tm == 0) stg[tj * kWarps + warp] = __fadd_rn(x2[tj * d + gw], comb);
        }
        __syncthreads();
        push_chunks(2 * n, [&](int c) { return stg + (c / 2) * kWarps + 4 * (c % 2); },
                    [&](int c) { return xs + (c / 2) * d + rank * kWarps + 4 * (c % 2); }, kFcXs);
        if (l + 1 < a.L) stage_experts(l + 1);  // this warp is done with layer l's rows
    }
    sync(kFcXs, a.L - 1);

    // Final RMSNorm of each wanted row (k_final_norm's order: 32-element warp sums added in order) for the vocab
    // kernel; clears its argmax key. CTA r writes output row r.
    const int out_rows = a.rows ? 1 : n;
    if (rank < out_rows && warp == 0) {
        int64_t src = rank;
        if (a.rows) src = checked_row(a.rows[0], n, true, a.err);
        const float* xr = xs + src * d;
        float tot = 0.f;
#pragma unroll
        for (int q = 0; q < 4; ++q) tot += warp_sum(fmaf(xr[q * 32 + lane], xr[q * 32 + lane], 0.f));
        const float inv = 1.0f / sqrtf(tot / float(d) + dm.eps);
        const float4 v = *reinterpret_cast<const float4*>(xr + lane * 4);
        *reinterpret_cast<float4*>(a.tf + size_t(rank) * d + lane * 4) =
            make_float4(__fmul_rn(__fmul_rn(v.x, inv), fnorm[0][0]), __fmul_rn(__fmul_rn(v.y, inv), fnorm[0][1]),
                        __fmul_rn(__fmul_rn(v.z, inv), fnorm[0][2]), __fmul_rn(__fmul_rn(v.w, inv), fnorm[0][3]));
        if (lane == 0 && a.keys) a.keys[rank] = 0ull;
    }
    cluster_sync_all();  // no CTA leaves while another may still store into it
}

}  // namespace cb200
