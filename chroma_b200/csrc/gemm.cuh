// bf16 GEMM on the sm_100a tensor cores: C[M, N] = A[M, K] . B[N, K]^T with fp32 accumulation in TMEM.
//
// Replaces the reference's cuBLAS SGEMM / scalar bf16 linear (chroma/_src/codegen/cuda/runtime.h:175-181,
// chroma/_src/codegen/gpu.py:263-273) and its per-(token, expert) einsum loops (gpu.py:390-424) for the GPT-OSS-20B/
// 120B-shaped programs. One kernel serves dense projections and grouped (per-expert) problems:
//
//   * persistent CTAs, one per SM, walk a static sequence of 128 x BN output tiles (no atomics);
//   * warp 0 (one thread) streams A and B tiles with TMA (128-byte swizzle) into a kGemmStages-deep ring;
//   * warp 1 allocates two BN-column TMEM accumulators and (one thread) issues tcgen05.mma (M=128, N=BN, K=16) per
//     64-wide K block, releasing each ring stage with tcgen05.commit and signalling the epilogue when a tile's
//     accumulation is done; tile i+1 accumulates into the other buffer while tile i is drained;
//   * warps 2-5 read the accumulator (each warp its 32-lane TMEM quadrant = 32 tile rows) with tcgen05.ld, apply the
//     fused epilogue (bias, rounding, residual add, SwiGLU) and store 16-byte row segments coalesced through a small
//     shared-memory stage, then hand the accumulator back.
//
// Grouped problems (MoE experts): rows [offsets[g], offsets[g+1]) of A multiply B rows [g*N, (g+1)*N); tiles never
// straddle groups (rows past a group's end are masked in the epilogue). All waits are bounded (tma.cuh).
#pragma once

#include "tcgen05.cuh"

namespace cb200 {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 192;
constexpr int kGemmMaxGroups = 256;

enum GemmEpi : int {
    kEpiStore = 0,    // C = round(acc + bias)
    kEpiResidual = 1, // C = round(R[row] + round(acc + bias))            (linear + residual, gpt_oss.py:209)
    kEpiSwiglu = 2,   // C[row, p] = swiglu(round(round(acc)+b) pairs)    (mlp1 + SwiGLU, gpt_oss.py:253-254)
    kEpiExpert = 3,   // C = round(round(acc) + bias[g])                   (mlp2 einsum + bias, gpt_oss.py:259-260)
    kEpiRope = 4,     // QKV + RoPE: q heads (C) and new K rows rotated, new V rows copied (gpt_oss.py:44-54, 189-202)
};

struct GemmArgs {
    int M, N, K;
    int epi;
    const __nv_bfloat16* bias;      // [groups][N] (group stride N), or nullptr
    const __nv_bfloat16* residual;  // [M][ldr] for kEpiResidual
    int ldr;
    __nv_bfloat16* C;               // [M][ldc]
    int ldc;
    float alpha, limit;             // SwiGLU slope and clamp
    int groups;                     // 1 for a dense GEMM
    const int* offsets;             // [groups + 1] row offsets of each group in A (device), or nullptr (dense)
    // Optional: A (and the offsets) are written by other GPUs; wait until each of wait_count flags reaches *wait_epoch
    // (expert-parallel dispatch) before reading them.
    const unsigned* wait_flags;
    int wait_count;
    const unsigned* wait_epoch;
    unsigned long long wait_timeout_ns;
    // Optional: greedy argmax keys per row (kEpiStore): the largest bf16 output, lowest column on ties (atomicMax of
    // argmax_key over each thread's columns of a tile; the caller zeroes the keys).
    unsigned long long* argmax_keys;
    int argmax_col_offset;  // added to the column index in the keys (a vocab shard's first global row)
    // Narrow last column tile (single-CTA kernel): when the last column tile holds at most half of BN columns, its
    // MMAs run at N = tail_n (those columns rounded up to 16) from a B tile of tail_n rows (the third tensor map), and
    // these tiles are scheduled after every full-width tile so they even out the per-SM totals. 0: full width.
    int tail_n;
    // kEpiRope (head_dim 64, single-CTA kernel): C is q [M][rope_H * 64]; output heads [rope_H, rope_H + rope_KV) go
    // rotated to rope_k and the next rope_KV heads unrotated to rope_v (rows of rope_KV * 64); rope_cs[row * 32 + j]
    // holds the rounded (cos, sin) of the row's position for frequency j.
    const float2* rope_cs;
    __nv_bfloat16* rope_k;
    __nv_bfloat16* rope_v;
    int rope_H, rope_KV;
    // Split-K (dense only): ksplit > 1 splits the K blocks over ksplit tiles whose raw fp32 sums go to
    // partial[ks][M][N]; k_gemm_splitk_epilogue then adds them in order and applies the epilogue.
    int ksplit;
    float* partial;
};

__device__ __forceinline__ float round_bf16(float x) { return bf16_round(x); }

// Epilogue staging: each epilogue warp owns 32 rows x 64 bytes of shared memory. 16-byte chunk c of row r sits at
// chunk c ^ ((r >> 1) & 3), so a row-per-thread write and an 8-rows-per-instruction coalesced read are both free of
// bank conflicts.
constexpr int kGemmStageBytes = 32 * 64;
__device__ __forceinline__ int stage_off(int r, int c) { return r * 64 + ((c ^ ((r >> 1) & 3)) << 4); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float swiglu_pair(float acc_g, float acc_l, float bg, float bl, float alpha, float limit) {
    const float hg = round_bf16(round_bf16(acc_g) + bg);
    const float hl = round_bf16(round_bf16(acc_l) + bl);
    const float glu = fminf(hg, limit);
    const float lin = fminf(fmaxf(hl, -limit), limit);
    const float z = round_bf16(glu * alpha);
    const float sg = round_bf16(fast_sigmoid_bf16in(z));  // z is a bf16 value: same bits as 1 / (1 + expf(-z))
    const float og = round_bf16(glu * sg);
    const float l1 = round_bf16(lin + 1.0f);
    return og * l1;
}

// Row-per-thread packed bf16 words -> stage -> coalesced 16-byte stores of rows [row_base, row_end).
// CHUNKS = 16-byte chunks per row (4 = 32 columns, 2 = 16 SwiGLU outputs).
template <int CHUNKS>
__device__ __forceinline__ void stage_store(__nv_bfloat16* C, int ldc, const uint32_t (&w)[16], int row_base,
                                            int row_end, int out_col, uint8_t* stage) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c)
        *reinterpret_cast<uint4*>(stage + stage_off(lane, c)) = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    __syncwarp();
#pragma unroll
    for (int pass = 0; pass < CHUNKS; ++pass) {
        const int r = pass * (32 / CHUNKS) + lane / CHUNKS, c = lane % CHUNKS;
        if (row_base + r < row_end)
            *reinterpret_cast<uint4*>(C + size_t(row_base + r) * ldc + out_col + 8 * c) =
                *reinterpret_cast<const uint4*>(stage + stage_off(r, c));
    }
    __syncwarp();
}

template <int CHUNKS>
__device__ __forceinline__ void stage_store(const GemmArgs& g, const uint32_t (&w)[16], int row_base, int row_end,
                                            int out_col, uint8_t* stage) {
    stage_store<CHUNKS>(g.C, g.ldc, w, row_base, row_end, out_col, stage);
}

// kEpiRope, one 64-wide head of an epilogue warp's 32 rows: `lo` and `hi` hold the accumulator columns [col0, col0 +
// 32) and [col0 + 32, col0 + 64) of row (row_base + lane). The values are rounded with the bias as in kEpiStore (the
// fused QKV linear), then q and K heads are rotated pairwise (lo[j], hi[j]) with the row's (cos, sin) of frequency j,
// each product and the sum rounded to bf16 as in k_rope_split; V heads pass unrotated. Stores go through `stage`.
__device__ __forceinline__ void gemm_rope_head(const GemmArgs& g, float (&lo)[32], float (&hi)[32],
                                               const __nv_bfloat16* bias, int row_base, int row_end, int col0,
                                               uint8_t* stage) {
    const int lane = threadIdx.x & 31;
    const int head = col0 >> 6;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        float bl[8], bh[8];
        if (bias) {
            const uint4 ul = __ldg(reinterpret_cast<const uint4*>(bias + col0) + c);
            const uint4 uh = __ldg(reinterpret_cast<const uint4*>(bias + col0 + 32) + c);
            const __nv_bfloat162* hl = reinterpret_cast<const __nv_bfloat162*>(&ul);
            const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&uh);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float2 fl = __bfloat1622float2(hl[j]), fh = __bfloat1622float2(hh[j]);
                bl[2 * j] = fl.x;
                bl[2 * j + 1] = fl.y;
                bh[2 * j] = fh.x;
                bh[2 * j + 1] = fh.y;
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) bl[j] = bh[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            lo[8 * c + j] = round_bf16(lo[8 * c + j] + bl[j]);
            hi[8 * c + j] = round_bf16(hi[8 * c + j] + bh[j]);
        }
    }
    if (head < g.rope_H + g.rope_KV) {
        const int row = min(row_base + lane, row_end - 1);  // rows past the end read a valid row and store nothing
        const float4* cs = reinterpret_cast<const float4*>(g.rope_cs + size_t(row) * 32);
#pragma unroll
        for (int p = 0; p < 16; ++p) {
            const float4 v = __ldg(cs + p);  // (cos, sin) of frequencies 2p and 2p + 1
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int j = 2 * p + u;
                const float c = u ? v.z : v.x, sn = u ? v.w : v.y;
                const float l = lo[j], h = hi[j];
                lo[j] = round_bf16(__fsub_rn(round_bf16(__fmul_rn(l, c)), round_bf16(__fmul_rn(h, sn))));
                hi[j] = round_bf16(__fadd_rn(round_bf16(__fmul_rn(h, c)), round_bf16(__fmul_rn(l, sn))));
            }
        }
    }
    __nv_bfloat16* dst;
    int ldc, col;
    if (head < g.rope_H) {
        dst = g.C;
        ldc = g.ldc;
        col = head * 64;
    } else if (head < g.rope_H + g.rope_KV) {
        dst = g.rope_k;
        ldc = g.rope_KV * 64;
        col = (head - g.rope_H) * 64;
    } else {
        dst = g.rope_v;
        ldc = g.rope_KV * 64;
        col = (head - g.rope_H - g.rope_KV) * 64;
    }
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(lo[2 * j], lo[2 * j + 1]);
    stage_store<4>(dst, ldc, w, row_base, row_end, col, stage);
#pragma unroll
    for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(hi[2 * j], hi[2 * j + 1]);
    stage_store<4>(dst, ldc, w, row_base, row_end, col + 32, stage);
}

// One 32-row x 32-column accumulator chunk of an epilogue warp: `v` holds row (row_base + lane), columns
// [col0, col0 + 32). Fast path (vec): 16-byte residual loads and output stores, coalesced through `stage`.
__device__ __forceinline__ void gemm_epilogue_chunk(const GemmArgs& g, const float (&v)[32], const __nv_bfloat16* bias,
                                                    int row_base, int row_end, int col0, bool vec, uint8_t* stage,
                                                    unsigned long long& best) {
    const int lane = threadIdx.x & 31;
    const int row = row_base + lane;
    if (vec && col0 + 32 <= g.N) {
        float b[32];
        if (bias) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 w = __ldg(reinterpret_cast<const uint4*>(bias + col0) + c);
                const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 f = __bfloat1622float2(h[j]);
                    b[8 * c + 2 * j] = f.x;
                    b[8 * c + 2 * j + 1] = f.y;
                }
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) b[j] = 0.f;
        }
        uint32_t w[16];
        if (g.epi == kEpiSwiglu) {
#pragma unroll
            for (int p = 0; p < 8; ++p)
                w[p] = pack_bf16x2(swiglu_pair(v[4 * p], v[4 * p + 1], b[4 * p], b[4 * p + 1], g.alpha, g.limit),
                                   swiglu_pair(v[4 * p + 2], v[4 * p + 3], b[4 * p + 2], b[4 * p + 3], g.alpha, g.limit));
            stage_store<2>(g, w, row_base, row_end, col0 / 2, stage);
        } else {
            float y[32];
#pragma unroll
            for (int j = 0; j < 32; ++j)
                y[j] = g.epi == kEpiExpert ? round_bf16(round_bf16(v[j]) + b[j]) : round_bf16(v[j] + b[j]);
            if (g.epi == kEpiResidual) {
                // Coalesced residual rows -> stage -> one row per thread.
#pragma unroll
                for (int pass = 0; pass < 4; ++pass) {
                    const int r = pass * 8 + (lane >> 2), c = lane & 3;
                    if (row_base + r < row_end)
                        *reinterpret_cast<uint4*>(stage + stage_off(r, c)) = *reinterpret_cast<const uint4*>(
                            g.residual + size_t(row_base + r) * g.ldr + col0 + 8 * c);
                }
                __syncwarp();
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint4 rw = *reinterpret_cast<const uint4*>(stage + stage_off(lane, c));
                    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&rw);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __bfloat1622float2(h[j]);
                        y[8 * c + 2 * j] = round_bf16(f.x + y[8 * c + 2 * j]);
                        y[8 * c + 2 * j + 1] = round_bf16(f.y + y[8 * c + 2 * j + 1]);
                    }
                }
                __syncwarp();
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) w[j] = pack_bf16x2(y[2 * j], y[2 * j + 1]);
            if (g.argmax_keys) {
#pragma unroll
                for (int j = 0; j < 32; ++j) best = max(best, argmax_key(y[j], g.argmax_col_offset + col0 + j));
            }
            stage_store<4>(g, w, row_base, row_end, col0, stage);
        }
        return;
    }
    // General path: ragged last columns or unaligned operands, one element at a time.
    if (row >= row_end) return;
    const int ncols = min(32, g.N - col0);
    if (g.epi == kEpiSwiglu) {
        __nv_bfloat16* out = g.C + size_t(row) * g.ldc + col0 / 2;
#pragma unroll
        for (int p = 0; p < 16; ++p) {
            if (2 * p + 1 >= ncols) break;
            const float bg = bias ? __bfloat162float(bias[col0 + 2 * p]) : 0.f;
            const float bl = bias ? __bfloat162float(bias[col0 + 2 * p + 1]) : 0.f;
            out[p] = __float2bfloat16_rn(swiglu_pair(v[2 * p], v[2 * p + 1], bg, bl, g.alpha, g.limit));
        }
        return;
    }
    __nv_bfloat16* out = g.C + size_t(row) * g.ldc + col0;
    const __nv_bfloat16* res = g.epi == kEpiResidual ? g.residual + size_t(row) * g.ldr + col0 : nullptr;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if (j >= ncols) break;
        const float b = bias ? __bfloat162float(bias[col0 + j]) : 0.f;
        float y = g.epi == kEpiExpert ? round_bf16(round_bf16(v[j]) + b) : round_bf16(v[j] + b);
        if (res) y = round_bf16(__bfloat162float(res[j]) + y);
        out[j] = __float2bfloat16_rn(y);
        if (g.argmax_keys) best = max(best, argmax_key(y, g.argmax_col_offset + col0 + j));
    }
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1) k_gemm_bf16(const __grid_constant__ CUtensorMap map_a,
                                                               const __grid_constant__ CUtensorMap map_b,
                                                               const __grid_constant__ CUtensorMap map_bt, GemmArgs g,
                                                               unsigned* err) {
    constexpr int A_BYTES = kGemmBM * kGemmBK * 2;
    constexpr int B_BYTES = BN * kGemmBK * 2;
    constexpr int STAGE = A_BYTES + B_BYTES;
    constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators: the epilogue drains one while the MMA fills the other
    extern __shared__ uint8_t gsm_raw[];
    uint8_t* gsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[kGemmStages], empty[kGemmStages], tmem_full[2], tmem_empty[2];
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;  // set by any role whose bounded wait gave up
    __shared__ int s_tiles[kGemmMaxGroups + 1];
    __shared__ int s_offsets[kGemmMaxGroups + 1];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ntiles_n = (g.N + BN - 1) / BN;
    const int kblocks = (g.K + kGemmBK - 1) / kGemmBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kGemmStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);
            mbar_init(&tmem_empty[a], 4);
        }
        abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&map_a);
        prefetch_tensormap(&map_b);
        if (g.tail_n) prefetch_tensormap(&map_bt);
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base, TMEM_COLS);
        tmem_relinquish();
    }
    // Weights and activations of this GEMM are produced by earlier kernels: wait before reading the offsets.
    pdl_wait();
    pdl_trigger();
    __syncthreads();  // barrier and abort_flag initialisation visible to every thread
    if (g.wait_flags && int(threadIdx.x) < g.wait_count &&
        !wait_flag_geq(g.wait_flags + threadIdx.x, *reinterpret_cast<const volatile unsigned*>(g.wait_epoch),
                       g.wait_timeout_ns, err))
        abort_flag = 1;  // published by the __syncthreads below, before any role starts
    for (int i = threadIdx.x; i <= g.groups; i += blockDim.x) s_offsets[i] = g.offsets ? g.offsets[i] : (i == 0 ? 0 : g.M);
    __syncthreads();
    if (warp == 0) {
        // s_tiles[grp] = sum over earlier groups of ceil(rows / 128): lane l scans groups [8l, 8l + 8), then the lanes'
        // totals are scanned across the warp (groups <= 256).
        int local[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int grp = lane * 8 + j;
            local[j] = sum;
            if (grp < g.groups) sum += (s_offsets[grp + 1] - s_offsets[grp] + kGemmBM - 1) / kGemmBM;
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (lane * 8 + j < g.groups) s_tiles[lane * 8 + j] = incl - sum + local[j];
        if (lane == 31) s_tiles[g.groups] = incl;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const int total_m = s_tiles[g.groups];
    const int ksplit = g.ksplit > 1 ? g.ksplit : 1;
    const int mn_tiles = total_m * ntiles_n;
    const int total = mn_tiles * ksplit;
    // Full-width tiles first (m-tile major), then one narrow tail tile per m-tile when g.tail_n is set.
    const int nfull = g.tail_n ? ntiles_n - 1 : ntiles_n;
    const int full_tiles = total_m * nfull;
    auto is_tail = [&](int t) { return g.tail_n && t % mn_tiles >= full_tiles; };
    const int kb_per = (kblocks + ksplit - 1) / ksplit;
    const uint32_t tmem = tmem_base;
    // Split-K part of tile t: K blocks [kb_lo, kb_hi).
    auto k_range = [&](int t, int& kb_lo, int& kb_hi) {
        const int ks = t / mn_tiles;
        kb_lo = ks * kb_per;
        kb_hi = min(kblocks, kb_lo + kb_per);
    };

    // Tile t -> (group, first row, row end, n0). Consecutive tiles share an m-tile (A reuse) and sweep the group's B.
    auto tile_of = [&](int t, int& grp, int& row0, int& row_end, int& n0) {
        t %= mn_tiles;
        int mt;
        if (t < full_tiles) {
            mt = t / nfull;
            n0 = (t % nfull) * BN;
        } else {
            mt = t - full_tiles;
            n0 = nfull * BN;
        }
        int lo = 0, hi = g.groups - 1;
        while (lo < hi) {  // last group with s_tiles[grp] <= mt
            const int mid = (lo + hi + 1) >> 1;
            if (s_tiles[mid] <= mt) lo = mid;
            else hi = mid - 1;
        }
        grp = lo;
        row0 = s_offsets[grp] + (mt - s_tiles[grp]) * kGemmBM;
        row_end = min(row0 + kGemmBM, s_offsets[grp + 1]);
    };

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;
            for (int t = blockIdx.x; t < total && !abort_flag; t += gridDim.x) {
                int grp, row0, row_end, n0, kb_lo, kb_hi;
                tile_of(t, grp, row0, row_end, n0);
                k_range(t, kb_lo, kb_hi);
                const bool tail = is_tail(t);
                for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
                    const int s = it % kGemmStages;
                    if (!mbar_wait(&empty[s], unsigned(((it / kGemmStages) & 1) ^ 1), err)) { abort_flag = 1; break; }
                    uint8_t* sa = gsm + size_t(s) * STAGE;
                    mbar_arrive_expect_tx(&full[s], tail ? A_BYTES + g.tail_n * kGemmBK * 2 : STAGE);
                    tma_load_2d(sa, &map_a, kb * kGemmBK, row0, &full[s]);
                    tma_load_2d(sa + A_BYTES, tail ? &map_bt : &map_b, kb * kGemmBK, grp * g.N + n0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_full = umma_idesc_bf16(kGemmBM, BN);
            const uint32_t idesc_tail = umma_idesc_bf16(kGemmBM, g.tail_n);
            int it = 0, tile_it = 0;
            for (int t = blockIdx.x; t < total && !abort_flag; t += gridDim.x, ++tile_it) {
                const int acc = tile_it & 1;
                const uint32_t idesc = is_tail(t) ? idesc_tail : idesc_full;
                if (!mbar_wait(&tmem_empty[acc], unsigned(((tile_it >> 1) & 1) ^ 1), err)) { abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d = tmem + uint32_t(acc * BN);
                int kb_lo, kb_hi;
                k_range(t, kb_lo, kb_hi);
                for (int kb = kb_lo; kb < kb_hi; ++kb, ++it) {
                    const int s = it % kGemmStages;
                    if (!mbar_wait(&full[s], unsigned((it / kGemmStages) & 1), err)) { abort_flag = 1; break; }
                    tc_fence_after();
                    const uint8_t* sa = gsm + size_t(s) * STAGE;
                    const uint64_t da = umma_desc_sw128(sa);
                    const uint64_t db = umma_desc_sw128(sa + A_BYTES);
#pragma unroll
                    for (int k = 0; k < kGemmBK / 16; ++k)  // advance 16 elements = 32 bytes = 2 in the >>4 field
                        umma_bf16(d, da + 2 * k, db + 2 * k, idesc, kb > kb_lo || k > 0);
                    umma_commit(&empty[s]);
                }
                if (abort_flag) break;
                umma_commit(&tmem_full[acc]);
            }
        }
    } else {
        // Epilogue warps 2..5: TMEM quadrant q = warp % 4 holds tile rows [32q, 32q + 32).
        const int q = warp & 3;
        uint8_t* stage = gsm + size_t(kGemmStages) * STAGE + size_t(q) * kGemmStageBytes;
        const bool vec = ((reinterpret_cast<uintptr_t>(g.C) | reinterpret_cast<uintptr_t>(g.residual) |
                           reinterpret_cast<uintptr_t>(g.bias)) & 15) == 0 &&
                         g.ldc % 8 == 0 && g.N % 8 == 0 && (g.epi != kEpiResidual || g.ldr % 8 == 0);
        int tile_it = 0;
        for (int t = blockIdx.x; t < total && !abort_flag; t += gridDim.x, ++tile_it) {
            const int acc = tile_it & 1;
            if (!mbar_wait(&tmem_full[acc], unsigned((tile_it >> 1) & 1), err)) { abort_flag = 1; break; }
            tc_fence_after();
            int grp, row0, row_end, n0;
            tile_of(t, grp, row0, row_end, n0);
            const __nv_bfloat16* bias = g.bias ? g.bias + size_t(grp) * g.N : nullptr;
            const uint32_t taddr = tmem + uint32_t(acc * BN) + (uint32_t(q * 32) << 16);
            unsigned long long best = 0ull;
            const int row = row0 + q * 32 + lane;
            if constexpr (BN % 64 == 0) {
                if (g.epi == kEpiRope) {  // whole heads: column chunk pairs
#pragma unroll 1
                    for (int c = 0; c < BN / 32; c += 2) {
                        const int col0 = n0 + c * 32;
                        if (col0 >= g.N) break;
                        float lo[32], hi[32];
                        tmem_load32(taddr + uint32_t(c * 32), lo);
                        tmem_load32(taddr + uint32_t(c * 32 + 32), hi);
                        gemm_rope_head(g, lo, hi, bias, row0 + q * 32, row_end, col0, stage);
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tmem_empty[acc]);
                    continue;
                }
            }
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                const int col0 = n0 + c * 32;
                if (col0 >= g.N) break;  // warp-uniform; a narrow tail tile wrote only its first tail_n columns
                float v[32];
                tmem_load32(taddr + uint32_t(c * 32), v);
                if (ksplit > 1) {  // raw partial sums; the split-K epilogue kernel finishes them
                    if (row < row_end) {
                        float* dst = g.partial + (size_t(t / mn_tiles) * g.M + row) * g.N + col0;
                        const int ncols = min(32, g.N - col0);
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < ncols) dst[j] = v[j];
                    }
                    continue;
                }
                gemm_epilogue_chunk(g, v, bias, row0 + q * 32, row_end, col0, vec, stage, best);
            }
            if (g.argmax_keys && ksplit == 1 && row < row_end && best) atomicMax(g.argmax_keys + row, best);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tmem_empty[acc]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// The same GEMM on CTA pairs (cta_group::2): a 2-CTA cluster computes 256 x 256 output tiles, each CTA streaming
// only its 128 rows of A and its 128 rows of B (32 KB per 64-wide K stage instead of 48 KB for the same MMA work
// per SM), so 6 stages fit in shared memory. The leader CTA issues the 256-row MMAs; each CTA drains its own 128 x
// 256 accumulator (two per CTA in TMEM, double-buffered) with the epilogue above. Dense and grouped; no split-K.
constexpr int kPairStages = 6;
constexpr int kPairBM = 256;  // rows per pair tile (128 per CTA)
constexpr int kPairBN = 256;  // columns per pair tile (each CTA loads 128 rows of B)
constexpr size_t kPairSmemBytes = size_t(kPairStages) * 2 * 128 * kGemmBK * 2 + 4 * kGemmStageBytes + 1024;

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    k_gemm_bf16_pair(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, GemmArgs g,
                     unsigned* err) {
    constexpr int HALF = 128 * kGemmBK * 2;  // one CTA's A (or B) rows of a stage
    constexpr int STAGE = 2 * HALF;
    constexpr uint32_t TMEM_COLS = 2 * kPairBN;
    extern __shared__ uint8_t psm_raw[];
    uint8_t* gsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(psm_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[kPairStages], empty[kPairStages], tmem_full[2], tmem_empty[2];
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    __shared__ int s_tiles[kGemmMaxGroups + 1];
    __shared__ int s_offsets[kGemmMaxGroups + 1];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    const int ntiles_n = (g.N + kPairBN - 1) / kPairBN;
    const int kblocks = (g.K + kGemmBK - 1) / kGemmBK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kPairStages; ++s) {
            mbar_init(&full[s], 1);   // the leader's expect_tx; both CTAs' bytes
            mbar_init(&empty[s], 1);  // one MMA commit per round
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tmem_full[a], 1);
            mbar_init(&tmem_empty[a], 8);  // leader only: 4 epilogue warps of each CTA
        }
        abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&map_a);
        prefetch_tensormap(&map_b);
    }
    if (warp == 1) {
        tmem_alloc_pair(&tmem_base, TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA signal
    tc_fence_after();
    pdl_wait();
    pdl_trigger();
    if (g.wait_flags && int(threadIdx.x) < g.wait_count &&
        !wait_flag_geq(g.wait_flags + threadIdx.x, *reinterpret_cast<const volatile unsigned*>(g.wait_epoch),
                       g.wait_timeout_ns, err))
        abort_flag = 1;
    for (int i = threadIdx.x; i <= g.groups; i += blockDim.x) s_offsets[i] = g.offsets ? g.offsets[i] : (i == 0 ? 0 : g.M);
    __syncthreads();
    if (warp == 0) {  // 256-row tiles per group, prefix-summed (as in k_gemm_bf16)
        int local[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int grp = lane * 8 + j;
            local[j] = sum;
            if (grp < g.groups) sum += (s_offsets[grp + 1] - s_offsets[grp] + kPairBM - 1) / kPairBM;
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (lane * 8 + j < g.groups) s_tiles[lane * 8 + j] = incl - sum + local[j];
        if (lane == 31) s_tiles[g.groups] = incl;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const int total = s_tiles[g.groups] * ntiles_n;
    const uint32_t tmem = tmem_base;

    auto tile_of = [&](int t, int& grp, int& row0, int& row_end, int& n0) {
        const int mt = t / ntiles_n;
        n0 = (t % ntiles_n) * kPairBN;
        int lo = 0, hi = g.groups - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_tiles[mid] <= mt) lo = mid;
            else hi = mid - 1;
        }
        grp = lo;
        row0 = s_offsets[grp] + (mt - s_tiles[grp]) * kPairBM;
        row_end = min(row0 + kPairBM, s_offsets[grp + 1]);
    };

    if (warp == 0) {
        if (lane == 0) {  // producer, both CTAs: own halves of A and B, counted on the leader's full barrier
            int it = 0;
            for (int t = cluster; t < total && !abort_flag; t += nclusters) {
                int grp, row0, row_end, n0;
                tile_of(t, grp, row0, row_end, n0);
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    if (!mbar_wait(&empty[s], unsigned(((it / kPairStages) & 1) ^ 1), err)) { abort_flag = 1; break; }
                    uint8_t* sa = gsm + size_t(s) * STAGE;
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * STAGE);
                    const uint32_t fb = cluster_addr(&full[s], 0);
                    tma_load_2d_pair(sa, &map_a, kb * kGemmBK, row0 + int(rank) * 128, fb);
                    tma_load_2d_pair(sa + HALF, &map_b, kb * kGemmBK, grp * g.N + n0 + int(rank) * 128, fb);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {  // MMA issue (leader only); commits go to both CTAs' barriers
            constexpr uint32_t idesc = umma_idesc_bf16(kPairBM, kPairBN);
            int it = 0, tile_it = 0;
            for (int t = cluster; t < total && !abort_flag; t += nclusters, ++tile_it) {
                const int acc = tile_it & 1;
                if (!mbar_wait(&tmem_empty[acc], unsigned(((tile_it >> 1) & 1) ^ 1), err)) { abort_flag = 1; break; }
                tc_fence_after();
                const uint32_t d = tmem + uint32_t(acc * kPairBN);
                for (int kb = 0; kb < kblocks; ++kb, ++it) {
                    const int s = it % kPairStages;
                    if (!mbar_wait(&full[s], unsigned((it / kPairStages) & 1), err)) { abort_flag = 1; break; }
                    tc_fence_after();
                    const uint8_t* sa = gsm + size_t(s) * STAGE;
                    const uint64_t da = umma_desc_sw128(sa);
                    const uint64_t db = umma_desc_sw128(sa + HALF);
#pragma unroll
                    for (int k = 0; k < kGemmBK / 16; ++k) umma_bf16_pair(d, da + 2 * k, db + 2 * k, idesc, kb > 0 || k > 0);
                    umma_commit_pair(cluster_addr(&empty[s], 0));
                    umma_commit_pair(cluster_addr(&empty[s], 1));
                }
                if (abort_flag) break;
                umma_commit_pair(cluster_addr(&tmem_full[acc], 0));
                umma_commit_pair(cluster_addr(&tmem_full[acc], 1));
            }
        }
    } else {
        // Epilogue warps 2..5 of each CTA: TMEM quadrant q = warp % 4 holds this CTA's tile rows [32q, 32q + 32).
        const int q = warp & 3;
        uint8_t* stage = gsm + size_t(kPairStages) * STAGE + size_t(q) * kGemmStageBytes;
        const bool vec = ((reinterpret_cast<uintptr_t>(g.C) | reinterpret_cast<uintptr_t>(g.residual) |
                           reinterpret_cast<uintptr_t>(g.bias)) & 15) == 0 &&
                         g.ldc % 8 == 0 && g.N % 8 == 0 && (g.epi != kEpiResidual || g.ldr % 8 == 0);
        int tile_it = 0;
        for (int t = cluster; t < total && !abort_flag; t += nclusters, ++tile_it) {
            const int acc = tile_it & 1;
            if (!mbar_wait(&tmem_full[acc], unsigned((tile_it >> 1) & 1), err)) { abort_flag = 1; break; }
            tc_fence_after();
            int grp, row0, row_end, n0;
            tile_of(t, grp, row0, row_end, n0);
            const int rbase = row0 + int(rank) * 128 + q * 32;
            const __nv_bfloat16* bias = g.bias ? g.bias + size_t(grp) * g.N : nullptr;
            const uint32_t taddr = tmem + uint32_t(acc * kPairBN) + (uint32_t(q * 32) << 16);
            unsigned long long best = 0ull;
#pragma unroll 1
            for (int c = 0; c < kPairBN / 32; ++c) {
                float v[32];
                tmem_load32(taddr + uint32_t(c * 32), v);
                const int col0 = n0 + c * 32;
                if (col0 >= g.N) continue;
                gemm_epilogue_chunk(g, v, bias, rbase, row_end, col0, vec, stage, best);
            }
            if (g.argmax_keys && rbase + lane < row_end && best) atomicMax(g.argmax_keys + rbase + lane, best);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(cluster_addr(&tmem_empty[acc], 0));
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, TMEM_COLS);
    }
}

// Split-K epilogue: C[r][c] from the ksplit partial sums (added in split order), with the kEpiStore or kEpiResidual
// epilogue of the GEMM and its argmax keys. grid = (ceil(N / 512), M); block = 256 (2 columns per thread).
__global__ void __launch_bounds__(256) k_gemm_splitk_epilogue(GemmArgs g) {
    __shared__ unsigned long long red[8];
    const int r = blockIdx.y;
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 2;
    pdl_wait();
    pdl_trigger();
    unsigned long long best = 0ull;
    if (c < g.N) {
        float a0 = 0.f, a1 = 0.f;
        for (int ks = 0; ks < g.ksplit; ++ks) {
            const float* p = g.partial + (size_t(ks) * g.M + r) * g.N + c;
            a0 += p[0];
            if (c + 1 < g.N) a1 += p[1];
        }
        const float b0 = g.bias ? __bfloat162float(g.bias[c]) : 0.f;
        const float b1 = g.bias && c + 1 < g.N ? __bfloat162float(g.bias[c + 1]) : 0.f;
        float y0 = round_bf16(a0 + b0), y1 = round_bf16(a1 + b1);
        if (g.epi == kEpiResidual) {
            y0 = round_bf16(__bfloat162float(g.residual[size_t(r) * g.ldr + c]) + y0);
            if (c + 1 < g.N) y1 = round_bf16(__bfloat162float(g.residual[size_t(r) * g.ldr + c + 1]) + y1);
        }
        __nv_bfloat16* out = g.C + size_t(r) * g.ldc + c;
        out[0] = __float2bfloat16_rn(y0);
        if (c + 1 < g.N) out[1] = __float2bfloat16_rn(y1);
        best = argmax_key(y0, g.argmax_col_offset + c);
        if (c + 1 < g.N) best = max(best, argmax_key(y1, g.argmax_col_offset + c + 1));
    }
    if (!g.argmax_keys) return;
    for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) best = max(best, red[w]);
        atomicMax(g.argmax_keys + r, max(best, red[0]));
    }
}

}  // namespace cb200
