// One-token decode step of a dev-sized GPT-OSS model (fp32 storage) through EVERY layer in one launch: a cluster
// of kDcC CTAs on kDcC SMs, the phases of each layer separated by hardware cluster barriers, activations exchanged
// through distributed shared memory. It replaces the per-layer chain k_attn_in -> k_attention -> k_out ->
// k_moe_up -> k_moe_down (5 dependent launches per layer, each a few microseconds of launch and drain latency
// around well under a microsecond of work) for the batch-1 decode program (chroma/_src/decoding/cached.py:22-60
// per step; the block of gpt_oss.py:189-265).
//
// Every CTA keeps its own copy of the small activations (residual x, x2, the QKV row, the attention output, the
// expert activations) in shared memory; a phase's outputs are split over the cluster's kDcC*kWarps warps and each
// result is stored into all kDcC copies (st.shared::cluster) before the barrier that ends the phase:
//
//   P1  RMSNorm (per CTA) -> QKV rows (2 per warp) -> +bias                 -> raw[]       barrier
//       RoPE on the gathered row (per CTA); CTA 0 stages the new K/V rows for the commit kernel
//   P2  attention over this CTA's ceil((ctx+1)/kDcC) keys (the K/V slices of every layer are copied into shared
//       memory by cp.async at the start), one warp per query head: (max, sum, P.V) partials -> parts[]    barrier
//       every CTA merges the kDcC partials of every head with the sink logit (split-KV softmax, cached.py:36-47)
//   P3  out-projection row (1 per warp) + bias + residual                   -> x2[]        barrier
//   P4  RMSNorm + gate + top-k + softmax (per CTA), then 4 (glu, linear) row pairs of the selected experts per
//       warp -> clamped SwiGLU                                                -> act[]       barrier
//   P5  mlp2 column (1 per warp) of each selected expert + bias, weighted combine in slot order + residual
//                                                                            -> x[]         barrier
//
// Weight rows a warp will use next are loaded into registers one phase ahead (the static QKV / out / gate rows of
// layer l+1 during P5 of layer l; the routed expert rows of P4 and P5 together, right after the routing), so the
// latency of the L2 reads overlaps the previous phase. The rounding points and summation orders of each dot
// product are those of the per-layer kernels (gptoss.cuh); only the attention's split over keys differs (kDcC
// chunks instead of 64-key chunks), as in any split-KV decode.
//
// Every CTA executes the same barrier sequence (no early exits), so the cluster barriers cannot wait on a CTA that
// left; the kernel has no spin-waits.
#pragma once

#include "flash.cuh"
#include "gptoss.cuh"
#include "tcgen05.cuh"

namespace cb200 {

constexpr int kDcC = 16;                 // CTAs per cluster (non-portable size: opted in at launch)
constexpr int kDcWarps = kDcC * kWarps;  // warps sharing each phase
constexpr int kDcRows1 = 2;              // QKV rows per warp
constexpr int kDcPairs = 4;              // (glu, linear) row pairs per warp
constexpr int kDcMaxK = 4;               // experts per token
constexpr int kDcMaxE = 2 * kWarps;      // gate rows (2 per warp)

struct DecodeClusterArgs {
    Dims dm;
    int L, ctx, kpc;                  // layers, cache rows, keys per CTA
    const LayerW<float>* layers;      // [L]
    const int* windows;               // [L] visible-window length per layer (ctx for full-attention layers)
    const float* emb;                 // [V][d]
    const float* final_norm;          // [d]
    const float* inv_freq;            // [hd/2]
    const int64_t* tokens;            // [1]
    const float* positions;           // [1]
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
};

// Shared-memory carve-up (in floats), identical on host and device.
struct DcLayout {
    int xs, xn, raw, qkv, parts, att, x2, gl, sidx, sw, inv, act, prow, kst, ks, vs, total;
    __host__ __device__ DcLayout(const Dims& dm, int L, int kpc) {
        auto up4 = [](int v) { return (v + 3) & ~3; };
        const int r1 = (dm.H + 2 * dm.KV) * dm.hd;
        int o = 0;
        xs = o; o += up4(dm.d);
        xn = o; o += up4(dm.d);
        raw = o; o += up4(r1);
        qkv = o; o += up4(r1);
        parts = o; o += up4(kDcC * dm.H * (dm.hd + 2));
        att = o; o += up4(dm.H * dm.hd);
        x2 = o; o += up4(dm.d);
        gl = o; o += up4(dm.E);
        sidx = o; o += 8;
        sw = o; o += 8;
        inv = o; o += 4;
        act = o; o += up4(dm.k * dm.I);
        prow = o; o += kWarps * 32;
        kst = o; o += up4(2 * kpc);  // int64 times of this CTA's cache rows
        ks = o; o += up4(L * kpc * dm.KV * dm.hd);
        vs = o; o += up4(L * kpc * dm.KV * dm.hd);
        total = o;
    }
};

__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Lanes 0..kDcC-1 store `v` (uniform over the warp) at `p`'s offset in CTA `lane` of the cluster.
__device__ __forceinline__ void cluster_broadcast(float* p, float v) {
    const int lane = threadIdx.x & 31;
    if (lane < kDcC) st_cluster_f32(cluster_addr(p, uint32_t(lane)), v);
}

// Warp dot product of one weight row held as NJ float4 per lane (elements lane*4 + 128*j) with a shared-memory row:
// per-lane FMA chain then the butterfly sum, the order of warp_gemv in gptoss.cuh.
template <int NJ>
__device__ __forceinline__ float dc_dot(const float (&w)[NJ][4], const float* x) {
    const int lane = threadIdx.x & 31;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const float4 v = *reinterpret_cast<const float4*>(x + lane * 4 + 128 * j);
        s = fmaf(w[j][0], v.x, s);
        s = fmaf(w[j][1], v.y, s);
        s = fmaf(w[j][2], v.z, s);
        s = fmaf(w[j][3], v.w, s);
    }
    return warp_sum(s);
}

template <int NJ>
__device__ __forceinline__ void dc_load(float (&w)[NJ][4], const float* row) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int j = 0; j < NJ; ++j) load4(row + lane * 4 + 128 * j, w[j]);
}

// out = x * (1/sqrt(mean(x^2) + eps)) * w over one row (the reduction order of rows_rmsnorm). Ends synchronised.
__device__ __forceinline__ void dc_norm(const float* x, float* out, int d, float eps, const float* __restrict__ w,
                                        float* inv) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 0) {
        float s = 0.f;
        for (int c = lane; c < d; c += 32) s = fmaf(x[c], x[c], s);
        s = warp_sum(s);
        if (lane == 0) *inv = 1.0f / sqrtf(s / float(d) + eps);
    }
    __syncthreads();
    const float iv = *inv;
    for (int c = threadIdx.x; c < d; c += blockDim.x) out[c] = __fmul_rn(__fmul_rn(x[c], iv), w[c]);
    __syncthreads();
}

// Per-warp weight rows of one layer that do not depend on the routing.
template <int NJ> struct DcStatic {
    float qkv[kDcRows1][NJ][4];
    float qkv_b[kDcRows1];
    float out[NJ][4];
    float out_b;
    float gate[2][NJ][4];
};

template <int NJ>
__device__ __forceinline__ void dc_load_static(DcStatic<NJ>& s, const LayerW<float>& w, const Dims& dm, int gw) {
    const int warp = threadIdx.x >> 5;
    const int r1 = (dm.H + 2 * dm.KV) * dm.hd;
#pragma unroll
    for (int u = 0; u < kDcRows1; ++u) {
        const int r = gw + kDcWarps * u;
        if (r < r1) {
            dc_load<NJ>(s.qkv[u], w.qkv_w + size_t(r) * dm.d);
            s.qkv_b[u] = w.qkv_b[r];
        }
    }
    if (gw < dm.d) {
        dc_load<NJ>(s.out, w.out_w + size_t(gw) * dm.H * dm.hd);
        s.out_b = w.out_b[gw];
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int e = warp + kWarps * u;
        if (e < dm.E) dc_load<NJ>(s.gate[u], w.gate_w + size_t(e) * dm.d);
    }
}

// NJ = d / 128 = H*hd / 128 = I / 128 (the host admits only such models).
template <int NJ>
__global__ void __launch_bounds__(kThreads, 1) k_decode_cluster(DecodeClusterArgs a) {
    extern __shared__ __align__(16) float dsm[];
    const Dims dm = a.dm;
    const DcLayout lay(dm, a.L, a.kpc);
    float* xs = dsm + lay.xs;
    float* xn = dsm + lay.xn;
    float* raw = dsm + lay.raw;
    float* qkv = dsm + lay.qkv;
    float* parts = dsm + lay.parts;
    float* att = dsm + lay.att;
    float* x2 = dsm + lay.x2;
    float* gl = dsm + lay.gl;
    int* sidx = reinterpret_cast<int*>(dsm + lay.sidx);
    float* sw = dsm + lay.sw;
    float* inv = dsm + lay.inv;
    float* act = dsm + lay.act;
    int64_t* kst = reinterpret_cast<int64_t*>(dsm + lay.kst);
    float* Ks = dsm + lay.ks;
    float* Vs = dsm + lay.vs;

    const int rank = int(cluster_ctarank());
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gw = rank * kWarps + warp;
    const int d = dm.d, hd = dm.hd, H = dm.H, KV = dm.KV, I = dm.I;
    const int r1 = (H + 2 * KV) * hd;
    const int row_kv = KV * hd;
    const int j0 = rank * a.kpc;                         // this CTA's first key
    const int nk = max(0, min(a.kpc, a.ctx + 1 - j0));   // its keys, the new token's included
    const int nkc = max(0, min(a.kpc, a.ctx - j0));      // of which cache rows

    DcStatic<NJ> st;
    dc_load_static<NJ>(st, a.layers[0], dm, gw);
    pdl_wait();
    pdl_trigger();

    // Cache slices of every layer (rows written by the previous step's commit, hence after the PDL wait).
    {
        const int row4 = row_kv / 4, per_layer = nkc * row4;
        for (int i = threadIdx.x; i < a.L * per_layer; i += blockDim.x) {
            const int l = i / per_layer, rem = i % per_layer, jj = rem / row4, c = (rem % row4) * 4;
            const size_t src = (size_t(l) * a.ctx + j0 + jj) * row_kv + c;
            const int dst = (l * a.kpc + jj) * row_kv + c;
            cp_async16(Ks + dst, a.cache_k + src);
            cp_async16(Vs + dst, a.cache_v + src);
        }
        cp_async_commit();
        for (int jj = threadIdx.x; jj < nkc; jj += blockDim.x) kst[jj] = a.slots[j0 + jj];
    }
    {
        const int64_t row = checked_row(a.tokens[0], dm.V, false, a.err);
        for (int c = threadIdx.x; c < d; c += blockDim.x) xs[c] = a.emb[size_t(row) * d + c];
    }
    const float pos = a.positions[0];
    const int64_t t_i = a.pos0[0];
    cp_async_wait<0>();
    __syncthreads();
    cluster_sync_all();  // every CTA of the cluster is running before the first remote store

    for (int l = 0; l < a.L; ++l) {
        const LayerW<float> w = a.layers[l];
        // ---- P1: norm, QKV rows, bias -> raw[] of every CTA
        dc_norm(xs, xn, d, dm.eps, w.attn_norm, inv);
#pragma unroll
        for (int u = 0; u < kDcRows1; ++u) {
            const int r = gw + kDcWarps * u;
            if (r < r1) {
                const float acc = dc_dot<NJ>(st.qkv[u], xn);
                cluster_broadcast(raw + r, __fadd_rn(acc, st.qkv_b[u]));
            }
        }
        cluster_sync_all();
        // RoPE of the q and k heads (gpt_oss.py:44-54), v heads copied; CTA 0 stages the new K/V rows.
        {
            const int half = hd / 2;
            for (int i = threadIdx.x; i < (H + 2 * KV) * half; i += blockDim.x) {
                const int h = i / half, j = i % half;
                const float lo = raw[h * hd + j], hi = raw[h * hd + j + half];
                float o1 = lo, o2 = hi;
                if (h < H + KV) {
                    const float angle = __fmul_rn(pos, a.inv_freq[j]);
                    float s, c;
                    sincosf(angle, &s, &c);
                    c = __fmul_rn(c, dm.conc);
                    s = __fmul_rn(s, dm.conc);
                    o1 = __fsub_rn(__fmul_rn(lo, c), __fmul_rn(hi, s));
                    o2 = __fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, s));
                }
                qkv[h * hd + j] = o1;
                qkv[h * hd + j + half] = o2;
                if (rank == 0 && h >= H) {
                    float* dst = h < H + KV ? a.new_k + size_t(l) * row_kv + (h - H) * hd
                                            : a.new_v + size_t(l) * row_kv + (h - H - KV) * hd;
                    dst[j] = o1;
                    dst[j + half] = o2;
                }
            }
        }
        __syncthreads();
        // ---- P2: attention partials over this CTA's keys, one warp per query head
        {
            const float* Kl = Ks + size_t(l) * a.kpc * row_kv;
            const float* Vl = Vs + size_t(l) * a.kpc * row_kv;
            const int window = a.windows[l];
            float* prow = dsm + lay.prow + warp * 32;
            const int groups = 32 / hd, g = lane / hd, dd = lane % hd;
            for (int hq = warp; hq < H; hq += kWarps) {
                const int kvh = hq / dm.G;
                const float* qv = qkv + hq * hd;
                float s = -INFINITY;
                if (lane < nk) {
                    const int j = j0 + lane;
                    const float* kr = j < a.ctx ? Kl + lane * row_kv + kvh * hd : qkv + (H + kvh) * hd;
                    float dot = 0.f;
                    for (int e = 0; e < hd; ++e) dot = fmaf(qv[e], kr[e], dot);
                    s = __fmul_rn(dot, dm.sm_scale);
                    const int64_t t_j = j < a.ctx ? kst[lane] : t_i;
                    const bool valid = j >= a.ctx || t_j >= 0;
                    const bool visible = valid && t_j <= t_i && (window <= 0 || t_j > t_i - window);
                    if (!visible) s = -INFINITY;
                }
                const float mx = warp_max(s);
                const float p = (lane < nk && mx != -INFINITY) ? expf(s - mx) : 0.f;
                const float lsum = warp_sum(p);
                prow[lane] = p;
                __syncwarp();
                float acc = 0.f;
                for (int jj = g; jj < nk; jj += groups) {
                    const int j = j0 + jj;
                    const float* vr = j < a.ctx ? Vl + jj * row_kv + kvh * hd : qkv + (H + KV + kvh) * hd;
                    acc = fmaf(prow[jj], vr[dd], acc);
                }
                for (int o = hd; o < 32; o <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
                const float ov = __shfl_sync(0xffffffffu, acc, (lane + 30) & 31);  // lane i <- o[i - 2]
                const float val = lane == 0 ? mx : (lane == 1 ? lsum : ov);
                if (lane < hd + 2) {
                    float* dst = parts + (rank * H + hq) * (hd + 2) + lane;
#pragma unroll 4
                    for (int r = 0; r < kDcC; ++r) st_cluster_f32(cluster_addr(dst, uint32_t(r)), val);
                }
                __syncwarp();
            }
        }
        cluster_sync_all();
        // Merge the kDcC partials of every head with its sink (the split-KV merge of k_attention).
        for (int hq = warp; hq < H; hq += kWarps) {
            const float sink = w.sinks[hq];
            float M = sink;
            for (int c = 0; c < kDcC; ++c) M = fmaxf(M, parts[(c * H + hq) * (hd + 2)]);
            float Lsum = expf(sink - M);
            for (int c = 0; c < kDcC; ++c) {
                const float mc = parts[(c * H + hq) * (hd + 2)];
                if (mc != -INFINITY) Lsum += parts[(c * H + hq) * (hd + 2) + 1] * expf(mc - M);
            }
            if (lane < hd) {
                float o = 0.f;
                for (int c = 0; c < kDcC; ++c) {
                    const float mc = parts[(c * H + hq) * (hd + 2)];
                    if (mc != -INFINITY) o += parts[(c * H + hq) * (hd + 2) + 2 + lane] * expf(mc - M);
                }
                att[hq * hd + lane] = o / Lsum;
            }
        }
        __syncthreads();
        // ---- P3: out-projection + bias + residual -> x2[]
        if (gw < d) {
            const float acc = dc_dot<NJ>(st.out, att);
            cluster_broadcast(x2 + gw, __fadd_rn(xs[gw], __fadd_rn(acc, st.out_b)));
        }
        cluster_sync_all();
        // ---- P4: norm, gate, top-k, softmax (every CTA), then the selected experts' mlp1 pairs -> act[]
        dc_norm(x2, xn, d, dm.eps, w.mlp_norm, inv);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int e = warp + kWarps * u;
            if (e < dm.E) {
                const float acc = dc_dot<NJ>(st.gate[u], xn);
                if (lane == 0) gl[e] = __fadd_rn(acc, w.gate_b[e]);
            }
        }
        __syncthreads();
        if (warp == 0) warp_topk_softmax<float>(gl, dm.E, dm.k, sidx, sw);
        __syncthreads();
        if (rank == 0 && a.routes && threadIdx.x < dm.k) a.routes[size_t(l) * dm.k + threadIdx.x] = sidx[threadIdx.x];
        float w1[kDcPairs][2][NJ][4], b1[kDcPairs][2];
        float w2[kDcMaxK][NJ][4], b2[kDcMaxK];
#pragma unroll
        for (int u = 0; u < kDcPairs; ++u) {
            const int P = gw + kDcWarps * u;
            if (P < dm.k * I) {
                const int s = P / I, p = P % I;
                const int e = int(checked_row(sidx[s], dm.E, true, a.err));
                const float* W1 = w.w1 + (size_t(e) * 2 * I + 2 * p) * d;
                dc_load<NJ>(w1[u][0], W1);
                dc_load<NJ>(w1[u][1], W1 + d);
                b1[u][0] = w.b1[size_t(e) * 2 * I + 2 * p];
                b1[u][1] = w.b1[size_t(e) * 2 * I + 2 * p + 1];
            }
        }
        if (gw < d) {
#pragma unroll
            for (int u = 0; u < kDcMaxK; ++u) {
                if (u < dm.k) {
                    const int e = int(checked_row(sidx[u], dm.E, true, a.err));
                    dc_load<NJ>(w2[u], w.w2 + (size_t(e) * d + gw) * I);
                    b2[u] = w.b2[size_t(e) * d + gw];
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kDcPairs; ++u) {
            const int P = gw + kDcWarps * u;
            if (P < dm.k * I) {
                const int s = P / I, p = P % I;
                const float hg = __fadd_rn(dc_dot<NJ>(w1[u][0], xn), b1[u][0]);
                const float hlin = __fadd_rn(dc_dot<NJ>(w1[u][1], xn), b1[u][1]);
                // Clamped SwiGLU (gpt_oss.py:212-219), the arithmetic of k_moe_up.
                const float glu = fminf(hg, dm.limit);
                const float lin = fminf(fmaxf(hlin, -dm.limit), dm.limit);
                const float z = __fmul_rn(glu, dm.alpha);
                const float sg = 1.0f / (1.0f + expf(-z));
                const float og = __fmul_rn(glu, sg);
                const float l1 = __fadd_rn(lin, 1.0f);
                cluster_broadcast(act + s * I + p, __fmul_rn(og, l1));
            }
        }
        cluster_sync_all();
        // ---- P5: mlp2 columns, weighted combine in slot order, residual -> x[]; next layer's static rows
        float xnew = 0.f;
        if (gw < d) {
            float comb = 0.f;
#pragma unroll
            for (int u = 0; u < kDcMaxK; ++u) {
                if (u < dm.k) {
                    const float part = dc_dot<NJ>(w2[u], act + u * I);
                    comb = __fadd_rn(comb, __fmul_rn(__fadd_rn(part, b2[u]), sw[u]));
                }
            }
            xnew = __fadd_rn(x2[gw], comb);
        }
        if (l + 1 < a.L) dc_load_static<NJ>(st, a.layers[l + 1], dm, gw);
        if (gw < d) cluster_broadcast(xs + gw, xnew);
        cluster_sync_all();
    }

    // Final RMSNorm of the token's row (gpt_oss.py:309) for the vocab kernel; clears the argmax key.
    if (rank == 0) {
        if (a.rows) checked_row(a.rows[0], 1, true, a.err);
        dc_norm(xs, a.tf, d, dm.eps, a.final_norm, inv);
        if (threadIdx.x == 0 && a.keys) a.keys[0] = 0ull;
    }
}

}  // namespace cb200
