// Flash attention for prefill chunks on the 5th-generation tensor cores (head_dim 64, bf16): the same sink attention
// as k_flash_prefill (chroma/models/gpt_oss.py:133-151, chroma/models/cached.py:36-47), with both products issued
// as tcgen05.mma into TMEM instead of mma.sync into registers.
//
// One CTA = two tiles of 128 query rows (256 consecutive rows) of one head of one sequence, which share every K and
// V tile; 10 warps:
//   warp 0 (one thread)  TMA: both Q tiles once, then K and V tiles of 64 keys into a kFtStages-deep ring, plus each
//                        tile's key positions (ring slots or chunk rows) written by the warp's lanes
//   warp 1 (one thread)  allocates 256 TMEM columns (S of query tile k at [64k, 64k + 64), O of query tile k at
//                        [128 + 64k, ...)) and issues, per key tile t, in ping-pong order:
//                          O0 += P0(t).V(t), S0(t+1) = Q0.K(t+1), O1 += P1(t).V(t), S1(t+1) = Q1.K(t+1)
//                        (M=128, N=64, K=64 each). P.V takes P straight from TMEM (the A operand of the
//                        tensor-memory form of tcgen05.mma) and V MN-major from its [key][dim] tile in shared memory.
//   warps 2-5, 6-9       the online softmax of query tile k = 0, 1, one query row per thread (TMEM lane = row):
//                        load the S row once (64 columns), mask, running max in the log2 domain, P = 2^(s - m)
//                        packed as bf16 pairs and stored over the first 32 columns of the same S (the columns this
//                        thread has already read), running sum; when the max grows, rescale the O row in TMEM; at the
//                        end O / (sum + sink term), stored as bf16
// P overwrites S in place, and the tensor core executes the MMAs of one issuing thread in order, so S_k(t+1) (written
// into the same columns) never lands before O_k += P_k(t).V(t) has read P_k(t); the commit that signals S_k(t+1) also
// covers that P.V, so the softmax may rescale O_k as soon as it sees S_k(t+1).
// While one warpgroup works on its softmax, the tensor core runs the other tile's products. The masking test is
// hoisted out of the per-element code (a 64-bit visibility word per row, applied only on tiles that need it): left
// inside the unrolled element loops it was predicated into every tile and took most of the ALU pipe. Tiles with no
// visible key are never loaded (ring tiles screened against the slot positions, own tiles from the window's edge),
// as in k_flash_prefill. 2 CTAs fit an SM (about 86 KB of shared memory and 256 TMEM columns each). All waits are
// bounded (tma.cuh).
#pragma once

#include "flash.cuh"
#include "tcgen05.cuh"

namespace cb200 {

constexpr int kFtRows = 128;   // query rows per query tile
constexpr int kFtQ = 2;        // query tiles per CTA
constexpr int kFtKeys = 64;    // keys per tile
constexpr int kFtStages = 3;   // K/V ring depth
constexpr int kFtThreads = 320;
constexpr int kFtMaxCacheTiles = 1024;
constexpr int kFtTile = kFtKeys * kFaDim * 2;  // one K or V tile: 8 KB
// Of each group of 4 (s, s') pairs of a row, the pairs with index kFtPolyFrom..3 take 2^x from exp2_poly (4: none; the
// special-function unit is not the limit at 2 CTAs per SM, and the polynomial costs issue slots).
constexpr int kFtPolyFrom = 4;
// Q 2 x 16 KB | K,V x kFtStages 16 KB | key positions 512 B per stage | live cache tiles 2 KB + bits 128 B, + alignment
constexpr size_t kFtSmemBytes = 1024 + kFtQ * kFtRows * kFaDim * 2 + 2 * kFtStages * size_t(kFtTile) +
                                kFtStages * kFtKeys * sizeof(int64_t) + kFtMaxCacheTiles * 2 + kFtMaxCacheTiles / 8;

struct FlashMaps {
    CUtensorMap q;       // [B*n][H][64]: box {64, 1, 128}
    CUtensorMap kn, vn;  // chunk rows [B*n][KV][64]: box {64, 1, 64}
    CUtensorMap kc, vc;  // ring cache of this layer [B][ctx][KV][64] (4-D): box {64, 1, 64, 1}
};

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
            "r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::
            "r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
        : "memory");
}

// Shared-memory descriptor of a 128-byte-swizzled tile read MN-major (rows of 64 elements along N, 8-row atoms of
// 1024 bytes along K): the V tile [key][dim] as the B operand of P.V.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(const void* smem_tile) {
    const uint64_t addr = smem_addr(smem_tile);
    uint64_t d = 0;
    d |= (addr >> 4) & 0x3FFFull;
    d |= uint64_t(8192 >> 4) << 16;   // LBO: next 64-element block along N (a single block here)
    d |= uint64_t(1024 >> 4) << 32;   // SBO: next 8 keys
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// D[tmem] (+)= A[tmem] * B[smem]: A (M rows on TMEM lanes, K-major, two bf16 per 32-bit column) read from tensor
// memory. Issued by a single thread.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(uint32_t(accumulate))
        : "memory");
}

// 32 lanes x 32 columns from TMEM without waiting (tmem_wait_ld() before the registers are read).
__device__ __forceinline__ void tmem_load32_async(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit words into TMEM; waits for the store to complete.
__device__ __forceinline__ void tmem_store32u(uint32_t taddr, const uint32_t* w) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7]), "r"(w[8]), "r"(w[9]),
        "r"(w[10]), "r"(w[11]), "r"(w[12]), "r"(w[13]), "r"(w[14]), "r"(w[15]), "r"(w[16]), "r"(w[17]), "r"(w[18]),
        "r"(w[19]), "r"(w[20]), "r"(w[21]), "r"(w[22]), "r"(w[23]), "r"(w[24]), "r"(w[25]), "r"(w[26]), "r"(w[27]),
        "r"(w[28]), "r"(w[29]), "r"(w[30]), "r"(w[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_store32(uint32_t taddr, const float (&v)[32]) {
    uint32_t w[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(v[i]);
    tmem_store32u(taddr, w);
}

// 2^x on the FMA pipe, for x <= 8 (the softmax's exponents): x = j + f with j = round(x) and f in [-1/2, 1/2] (the
// rounding by adding and subtracting 1.5 * 2^23), 2^f from a cubic with constant term 1 fitted here for the least
// maximum relative error on [-1/2, 1/2] (1.0e-4, far below the half unit of the bf16 that P is rounded to), and
// 2^j added to the exponent field. x below -126 gives 2^-126 or less (the caller's sums do not see it); -inf gives 0.
__device__ __forceinline__ float exp2_poly(float x) {
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
    const float xc = fmaxf(x, -126.0f);
    const float t = xc + kRound;
    const float f = xc - (t - kRound);
    float p = fmaf(0.05500858277082443f, f, 0.24221037328243256f);
    p = fmaf(p, f, 0.6932829022407532f);
    p = fmaf(p, f, 1.0f);
    const float y = __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
    return x == -INFINITY ? 0.0f : y;
}

// Packed pairs of fp32 (the f32x2 instructions of sm_100): lo in the low word.
__device__ __forceinline__ uint64_t f32x2(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f32x2_split(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// exp2_poly on a packed pair, the arithmetic in f32x2 (same rounding per element as exp2_poly).
__device__ __forceinline__ void exp2_poly2(uint64_t x2, float& ya, float& yb) {
    constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
    float xa, xb;
    f32x2_split(x2, xa, xb);
    const uint64_t xc = f32x2(fmaxf(xa, -126.0f), fmaxf(xb, -126.0f));
    const uint64_t t = fadd2(xc, f32x2(kRound, kRound));
    const uint64_t f = fsub2(xc, fsub2(t, f32x2(kRound, kRound)));
    uint64_t p = ffma2(f32x2(0.05500858277082443f, 0.05500858277082443f), f,
                       f32x2(0.24221037328243256f, 0.24221037328243256f));
    p = ffma2(p, f, f32x2(0.6932829022407532f, 0.6932829022407532f));
    p = ffma2(p, f, f32x2(1.0f, 1.0f));
    float pa, pb, ta, tb;
    f32x2_split(p, pa, pb);
    f32x2_split(t, ta, tb);
    ya = xa == -INFINITY ? 0.0f : __uint_as_float(__float_as_uint(pa) + (__float_as_uint(ta) << 23));
    yb = xb == -INFINITY ? 0.0f : __uint_as_float(__float_as_uint(pb) + (__float_as_uint(tb) << 23));
}

// grid = (ceil(n / 256), H, B); block = kFtThreads; dynamic shared memory kFtSmemBytes.
__global__ void __launch_bounds__(kFtThreads, 2) k_flash_prefill_tc(const __grid_constant__ FlashMaps maps, FlashArgs a,
                                                                    const __nv_bfloat16* __restrict__ sinks,
                                                                    __nv_bfloat16* __restrict__ out, unsigned* err) {
    extern __shared__ uint8_t ft_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ft_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* Qs = sm;                                      // [2][128][64] SW128
    uint8_t* KV = Qs + kFtQ * kFtRows * kFaDim * 2;        // stage s: K at KV + 2s*tile, V at KV + (2s+1)*tile
    int64_t* tpos = reinterpret_cast<int64_t*>(KV + 2 * kFtStages * kFtTile);  // [kFtStages][64] key positions
    uint16_t* live_list = reinterpret_cast<uint16_t*>(tpos + kFtStages * kFtKeys);
    uint32_t* live_bits = reinterpret_cast<uint32_t*>(live_list + kFtMaxCacheTiles);
    __shared__ uint64_t q_full, kv_full[kFtStages], kv_empty[kFtStages], s_full[kFtQ], p_full[kFtQ], pv_done[kFtQ];
    __shared__ uint32_t tmem_base;
    __shared__ int s_nlive;
    __shared__ volatile int abort_flag;

    const int qb = gridDim.x - 1 - blockIdx.x;  // heavy (late) query blocks first
    const int h = blockIdx.y, b = blockIdx.z;
    const int kvh = h / a.G;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int i0 = qb * kFtQ * kFtRows;
    const int i_last = min(i0 + kFtQ * kFtRows, a.n) - 1;
    const int cache_tiles = (a.ctx + kFtKeys - 1) / kFtKeys;

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int s = 0; s < kFtStages; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int k = 0; k < kFtQ; ++k) {
            mbar_init(&s_full[k], 1);
            mbar_init(&p_full[k], 4);  // the 4 softmax warps of query tile k
            mbar_init(&pv_done[k], 1);
        }
        abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&maps.q);
        prefetch_tensormap(&maps.kn);
        prefetch_tensormap(&maps.vn);
        if (a.ctx) {
            prefetch_tensormap(&maps.kc);
            prefetch_tensormap(&maps.vc);
        }
    }
    for (int w = threadIdx.x; w < (cache_tiles + 31) / 32; w += blockDim.x) live_bits[w] = 0;
    if (warp == 1) {
        tmem_alloc(&tmem_base, 256);
        tmem_relinquish();
    }
    pdl_wait();
    pdl_trigger();
    const int64_t p0 = a.pos0 ? a.pos0[b] : 0;
    const int64_t first = p0 + i0, last = p0 + i_last;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Screen the ring: a cache tile is live when one of its slots holds a position some row of the block can see.
    for (int j = threadIdx.x; j < a.ctx; j += blockDim.x) {
        const int64_t tj = a.slots[size_t(b) * a.ctx + j];
        if (tj >= 0 && tj <= last && (a.window <= 0 || tj > first - a.window))
            atomicOr(&live_bits[(j / kFtKeys) >> 5], 1u << ((j / kFtKeys) & 31));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int nl = 0;
        for (int w = 0; w < (cache_tiles + 31) / 32; ++w) {
            uint32_t bits = live_bits[w];
            while (bits) {
                const int bit = __ffs(bits) - 1;
                bits &= bits - 1;
                live_list[nl++] = uint16_t(w * 32 + bit);
            }
        }
        s_nlive = nl;
    }
    __syncthreads();
    const int nlive = s_nlive;
    const int own_lo = a.window > 0 ? max(0, i0 - a.window + 1) / kFtKeys : 0;
    const int own_hi = (i_last + kFtKeys) / kFtKeys;
    const int tiles = nlive + max(0, own_hi - own_lo);
    const uint32_t tmem = tmem_base;
    auto tile_key0 = [&](int tile, bool& cached) {
        cached = tile < nlive;
        return (cached ? int(live_list[tile]) : own_lo + tile - nlive) * kFtKeys;
    };

    if (warp == 0) {
        // ---- producer: both Q tiles once, then K/V tiles and their key positions
        if (lane == 0) {
            mbar_arrive_expect_tx(&q_full, kFtQ * kFtRows * kFaDim * 2);
            for (int k = 0; k < kFtQ; ++k)
                tma_load_3d(Qs + size_t(k) * kFtRows * kFaDim * 2, &maps.q, 0, h, b * a.n + i0 + k * kFtRows, &q_full);
        }
        for (int t = 0; t < tiles && !abort_flag; ++t) {
            const int s = t % kFtStages;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&kv_empty[s], unsigned(((t / kFtStages) & 1) ^ 1), err);
            ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
            if (!ok) {
                if (lane == 0) abort_flag = 1;
                break;
            }
            bool cached;
            const int j0 = tile_key0(t, cached);
            const int limit = cached ? a.ctx : a.n;
            for (int c = lane; c < kFtKeys; c += 32) {
                const int j = j0 + c;
                tpos[s * kFtKeys + c] = j < limit ? (cached ? a.slots[size_t(b) * a.ctx + j] : p0 + j) : -1;
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive_expect_tx(&kv_full[s], 2 * kFtTile);
                uint8_t* Kd = KV + size_t(2 * s) * kFtTile;
                uint8_t* Vd = KV + size_t(2 * s + 1) * kFtTile;
                if (cached) {
                    tma_load_4d(Kd, &maps.kc, 0, kvh, j0, b, &kv_full[s]);
                    tma_load_4d(Vd, &maps.vc, 0, kvh, j0, b, &kv_full[s]);
                } else {
                    tma_load_3d(Kd, &maps.kn, 0, kvh, b * a.n + j0, &kv_full[s]);
                    tma_load_3d(Vd, &maps.vn, 0, kvh, b * a.n + j0, &kv_full[s]);
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issue, ping-pong over the two query tiles
        if (lane == 0) {
            constexpr uint32_t idesc_s = umma_idesc_bf16(kFtRows, kFtKeys);
            constexpr uint32_t idesc_o = umma_idesc_bf16(kFtRows, kFaDim) | (1u << 16);  // B (V) MN-major
            if (!mbar_wait(&q_full, 0, err)) abort_flag = 1;
            tc_fence_after();
            // S_k(u) = Q_k . K(u) into query tile k's S columns (K of tile u has landed: waited by the caller).
            auto issue_s = [&](int k, int u) {
                const uint64_t dq = umma_desc_sw128(Qs + size_t(k) * kFtRows * kFaDim * 2);
                const uint64_t dk = umma_desc_sw128(KV + size_t(2 * (u % kFtStages)) * kFtTile);
#pragma unroll
                for (int kk = 0; kk < kFaDim / 16; ++kk)
                    umma_bf16(tmem + uint32_t(k * kFtKeys), dq + 2 * kk, dk + 2 * kk, idesc_s, kk > 0);
                umma_commit(&s_full[k]);
            };
            auto wait_kv = [&](int u) {
                if (!mbar_wait(&kv_full[u % kFtStages], unsigned((u / kFtStages) & 1), err)) return false;
                tc_fence_after();
                return true;
            };
            if (tiles > 0 && !abort_flag) {
                if (wait_kv(0)) {
                    issue_s(0, 0);
                    issue_s(1, 0);
                } else {
                    abort_flag = 1;
                }
            }
            for (int t = 0; t < tiles && !abort_flag; ++t) {
                const int s = t % kFtStages;
                const uint64_t dv = umma_desc_sw128_mn(KV + size_t(2 * s + 1) * kFtTile);
                bool next_ready = false;
                for (int k = 0; k < kFtQ; ++k) {
                    // Query tile k's softmax has stored P_k(t) over S_k(t).
                    if (!mbar_wait(&p_full[k], unsigned(t & 1), err)) { abort_flag = 1; break; }
                    tc_fence_after();
                    const uint32_t tP = tmem + uint32_t(k * kFtKeys);
                    const uint32_t tO = tmem + uint32_t(2 * kFtKeys + k * kFaDim);
#pragma unroll
                    for (int kk = 0; kk < kFtKeys / 16; ++kk)  // 16 keys per step: 8 columns of P, +2 KB down V
                        umma_bf16_ts(tO, tP + 8 * kk, dv + 128 * kk, idesc_o, t > 0 || kk > 0);
                    if (t == tiles - 1) umma_commit(&pv_done[k]);
                    if (k == kFtQ - 1) umma_commit(&kv_empty[s]);
                    if (t + 1 < tiles) {
                        if (k == 0) {
                            if (!wait_kv(t + 1)) { abort_flag = 1; break; }
                            next_ready = true;
                        }
                        if (next_ready) issue_s(k, t + 1);
                    }
                }
            }
        }
    } else {
        // ---- softmax of query tile k: warp q (= warp % 4) owns TMEM lanes / tile rows [32q, 32q + 32)
        const int k = (warp - 2) >> 2;
        const int q = warp & 3;
        const int r = q * 32 + lane;  // this thread's query row within its tile
        const int i = i0 + k * kFtRows + r;
        const int ik0 = i0 + k * kFtRows, ik_last = min(ik0 + kFtRows, a.n) - 1;
        const int64_t ti = p0 + i;
        const bool row_ok = i < a.n;
        const uint32_t lane_base = uint32_t(q * 32) << 16;
        const uint32_t tS = tmem + uint32_t(k * kFtKeys) + lane_base;
        const uint32_t tO = tmem + uint32_t(2 * kFtKeys + k * kFaDim) + lane_base;
        float m_run = -INFINITY, l_run = 0.f;
        for (int t = 0; t < tiles && !abort_flag; ++t) {
            const int s = t % kFtStages;
            bool cached;
            const int j0 = tile_key0(t, cached);
            const bool masked = cached || j0 + kFtKeys - 1 > ik0 || (a.window > 0 && j0 <= ik_last - a.window);
            // S_k(t) has landed (and with it every earlier MMA, the last P_k.V included); the key positions of a
            // masked tile come with its K/V stage.
            if (!mbar_wait(&s_full[k], unsigned(t & 1), err) ||
                (masked && !mbar_wait(&kv_full[s], unsigned((t / kFtStages) & 1), err))) {
                abort_flag = 1;
                break;
            }
            tc_fence_after();
            uint32_t sv[64];
            tmem_load32_async(tS, sv);
            tmem_load32_async(tS + 32, sv + 32);
            tmem_wait_ld();
            // Masked keys get s = -inf (so max ignores them and 2^-inf = 0). The test is hoisted out of the
            // element loops: ring tiles compare slot positions, chunk tiles an index range.
            if (masked) {
                uint64_t vis = 0;  // bit e: key j0 + e visible to this row
                if (cached) {
#pragma unroll 4
                    for (int e = 0; e < kFtKeys; ++e) {
                        const int64_t tj = tpos[s * kFtKeys + e];
                        if (row_ok && tj >= 0 && tj <= ti && (a.window <= 0 || tj > ti - a.window))
                            vis |= 1ull << e;
                    }
                } else {
                    // chunk key j0 + e is visible to row i iff i - window < j0 + e <= i: bits [lo, hi]
                    const int hi = min(i - j0, kFtKeys - 1);
                    const int lo = a.window > 0 ? max(i - a.window + 1 - j0, 0) : 0;
                    vis = hi < lo ? 0ull : ((~0ull >> (63 - hi)) & (~0ull << lo));
                }
#pragma unroll
                for (int e = 0; e < kFtKeys; ++e)
                    if (!((vis >> e) & 1)) sv[e] = __float_as_uint(-INFINITY);
            }
            float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int e = 0; e < kFtKeys; e += 8) {
                mq[0] = fmax3(mq[0], __uint_as_float(sv[e]), __uint_as_float(sv[e + 1]));
                mq[1] = fmax3(mq[1], __uint_as_float(sv[e + 2]), __uint_as_float(sv[e + 3]));
                mq[2] = fmax3(mq[2], __uint_as_float(sv[e + 4]), __uint_as_float(sv[e + 5]));
                mq[3] = fmax3(mq[3], __uint_as_float(sv[e + 6]), __uint_as_float(sv[e + 7]));
            }
            const float mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
            // Lazy rescaling: the reference max moves only when the tile's max exceeds it by more than 8 (log2
            // domain), so P stays below 2^8 and most tiles leave O untouched; the sum uses the same reference, so the
            // result is unchanged.
            const float m_tile = mx * a.scale_log2;
            const float m_new = (m_run == -INFINITY || m_tile > m_run + 8.f) ? fmaxf(m_run, m_tile) : m_run;
            const bool none = m_new == -INFINITY;
            const float corr = none ? 1.f : fast_exp2(m_run - m_new);
            const float neg = none ? 0.f : -m_new;
            // P = 2^(s * scale - m) (masked keys: 2^-inf = 0), as bf16 pairs over S's first 32 columns; the exponent
            // arguments and the row sum in packed pairs (f32x2), four partial sums.
            float rs = 0.f;
            uint32_t pw[32];
#pragma unroll
            for (int u = 0; u < kFtKeys / 2; ++u) {
                const float xa = fmaf(__uint_as_float(sv[2 * u]), a.scale_log2, neg);
                const float xb = fmaf(__uint_as_float(sv[2 * u + 1]), a.scale_log2, neg);
                const bool poly = (u & 3) >= kFtPolyFrom;
                const float pa = poly ? exp2_poly(xa) : fast_exp2(xa);
                const float pb = poly ? exp2_poly(xb) : fast_exp2(xb);
                rs += pa + pb;
                pw[u] = pack_bf16(pa, pb);
            }
            tmem_store32u(tS, pw);
            if (t > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    float ov[32];
                    tmem_load32(tO + c * 32, ov);
#pragma unroll
                    for (int e = 0; e < 32; ++e) ov[e] *= corr;
                    tmem_store32(tO + c * 32, ov);
                }
            }
            l_run = l_run * corr + rs;
            m_run = m_new;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[k]);
        }
        // Final: wait for the last P_k.V, then O / (l + sink term) for this row.
        if (tiles > 0 && !abort_flag && mbar_wait(&pv_done[k], 0, err)) {
            tc_fence_after();
            float ov[2][32];
            tmem_load32(tO, ov[0]);
            tmem_load32(tO + 32, ov[1]);
            if (row_ok) {
                const float sink = __bfloat162float(sinks[h]) * 1.4426950408889634f;
                const float mf = fmaxf(m_run, sink);
                const float c = m_run == -INFINITY ? 0.f : exp2f(m_run - mf);
                const float inv = 1.0f / (l_run * c + exp2f(sink - mf));
                __nv_bfloat16* orow = out + ((size_t(b) * a.n + i) * a.H + h) * kFaDim;
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    uint32_t w4[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int e = ch * 8 + 2 * u;
                        w4[u] = pack_bf16(ov[e >> 5][e & 31] * c * inv, ov[(e + 1) >> 5][(e + 1) & 31] * c * inv);
                    }
                    *reinterpret_cast<uint4*>(orow + ch * 8) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// ---------------------------------------------------------------------------------------------------------------
// Flash decoding with TMA staging: the attention of k_flash_decode (n * G <= 16 query rows of one KV head against
// the ring cache, split over the keys, mma.sync on the packed GQA rows), with the K/V tiles brought in by one
// producer warp through the tensor maps into a kFdtStages-deep ring of mbarrier-tracked stages. The consumer warps
// release a stage with one arrival each instead of a CTA barrier per tile, and the bytes in flight per CTA are the
// ring's depth, not the loads its threads can issue. The M = 16 rows leave the 128-row tcgen05 tile mostly empty;
// the products are a small share of this kernel, which streams the cache.
//
// grid = (B, KV, splits); block = kFdtThreads (warps 0-3 consumers, warp 4 producer); dynamic shared memory
// kFdtSmemBytes: 4 CTAs per SM with 3 stages each (at C5's shape 65 us per layer against 78 us for the cp.async
// kernel; 6 stages at 2 CTAs per SM took 91 us: each CTA's tiles go through its 4 consumer warps one after another,
// so the tiles in flight per SM, not the bytes, set the pace). Each 64-key tile is 16 KB; tiles past the ring's end
// read the tensor map's zero fill, keys outside the split or the chunk are masked through their positions (-1).
// All waits are bounded.
constexpr int kFdtStages = 3;
constexpr int kFdtThreads = 160;
constexpr int kFdtTile = kFdKeys * kFaDim * 2;  // 8 KB: one K or V tile
constexpr size_t kFdtSmemBytes = 1024 + 2 * size_t(kFdtStages) * kFdtTile + size_t(kFdRows) * kFaDim * 2 +
                                 size_t(kFdtStages) * kFdKeys * sizeof(int64_t);

__global__ void __launch_bounds__(kFdtThreads, 4) k_flash_decode_tma(const __grid_constant__ FlashMaps maps,
                                                                  const __nv_bfloat16* __restrict__ q, DecodeArgs a,
                                                                  const __nv_bfloat16* __restrict__ sinks,
                                                                  __nv_bfloat16* __restrict__ out, unsigned* err) {
    extern __shared__ uint8_t fdt_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fdt_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* ring = sm;  // stage s: K at 2s tiles, V at 2s + 1 (128-byte swizzle, fa_swz order)
    __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(ring + 2 * size_t(kFdtStages) * kFdtTile);
    int64_t* ts0 = reinterpret_cast<int64_t*>(Qs + kFdRows * kFaDim);
    __shared__ uint64_t full[kFdtStages], empty[kFdtStages];
    __shared__ bool s_last;
    __shared__ volatile int abort_flag;

    const int b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int rows = a.n * a.G;  // real query rows (<= 16)
    if (threadIdx.x == 0) {
        for (int st = 0; st < kFdtStages; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], 4);  // the 4 consumer warps
        }
        abort_flag = 0;
        fence_barrier_init();
        prefetch_tensormap(&maps.kc);
        prefetch_tensormap(&maps.vc);
        prefetch_tensormap(&maps.kn);
        prefetch_tensormap(&maps.vn);
    }
    pdl_wait();
    pdl_trigger();
    const int64_t p0 = a.pos0[b];
    // Q rows: row r = i * G + gh is query row i of head kvh * G + gh (rows >= n * G are zero).
    for (int e = threadIdx.x; e < kFdRows * 8; e += blockDim.x) {
        const int r = e >> 3, c = (e & 7) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < rows) {
            const int i = r / a.G, h = kvh * a.G + r % a.G;
            v = *reinterpret_cast<const uint4*>(q + ((size_t(b) * a.n + i) * a.H + h) * kFaDim + c);
        }
        *reinterpret_cast<uint4*>(Qs + fa_swz(r, c)) = v;
    }
    __syncthreads();
    const int j_begin = split * a.split_keys, j_end = min(a.ctx, j_begin + a.split_keys);
    const int cache_tiles = j_end > j_begin ? (j_end - j_begin + kFdKeys - 1) / kFdKeys : 0;
    const bool own = split == a.splits - 1;
    const int tiles = cache_tiles + (own ? 1 : 0);  // n <= 16 < 64: the own rows fit one tile

    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

    if (warp == 4) {
        // ---- producer: positions by the warp's lanes, the two tiles by lane 0
        for (int t = 0; t < tiles && !abort_flag; ++t) {
            const int st = t % kFdtStages;
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&empty[st], unsigned(((t / kFdtStages) & 1) ^ 1), err);
            if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) {
                if (lane == 0) abort_flag = 1;
                break;
            }
            const bool cached = t < cache_tiles;
            const int j0 = cached ? j_begin + t * kFdKeys : 0;
            const int limit = cached ? j_end : a.n;
            for (int c = lane; c < kFdKeys; c += 32) {
                const int j = j0 + c;
                ts0[st * kFdKeys + c] = j < limit ? (cached ? a.slots[size_t(b) * a.ctx + j] : p0 + j) : -1;
            }
            __syncwarp();
            if (lane == 0) {
                uint8_t* Kd = ring + size_t(2 * st) * kFdtTile;
                uint8_t* Vd = Kd + kFdtTile;
                mbar_arrive_expect_tx(&full[st], 2 * kFdtTile);
                if (cached) {
                    tma_load_4d(Kd, &maps.kc, 0, kvh, j0, b, &full[st]);
                    tma_load_4d(Vd, &maps.vc, 0, kvh, j0, b, &full[st]);
                } else {
                    tma_load_3d(Kd, &maps.kn, 0, kvh, b * a.n, &full[st]);
                    tma_load_3d(Vd, &maps.vn, 0, kvh, b * a.n, &full[st]);
                }
            }
        }
    } else {
        // ---- consumers: warp w takes keys [16w, 16w + 16) of every tile with its own online softmax
        int64_t t_row[2];  // this thread's rows g and g + 8: their positions (-1 marks a padding row)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int r = g + 8 * rr;
            t_row[rr] = r < rows ? p0 + r / a.G : -1;
        }
        uint32_t qf[4][4];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
            const int col = kk * 16 + 8 * (lane >> 4);
            ldsm_x4(qf[kk], Qs + fa_swz(row, col));
        }
        const int kw = warp * 16;
        for (int t = 0; t < tiles && !abort_flag; ++t) {
            const int st = t % kFdtStages;
            if (!mbar_wait(&full[st], unsigned((t / kFdtStages) & 1), err)) {
                abort_flag = 1;
                break;
            }
            const __nv_bfloat16* Kb = reinterpret_cast<const __nv_bfloat16*>(ring + size_t(2 * st) * kFdtTile);
            const __nv_bfloat16* Vb = Kb + kFdKeys * kFaDim;
            const int64_t* ts = ts0 + st * kFdKeys;
            float sc[2][4];
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                uint32_t kf[4];
                const int key = kw + (lane & 7) + 8 * (lane >> 4);
                const int col = kk * 16 + 8 * ((lane >> 3) & 1);
                ldsm_x4(kf, Kb + fa_swz(key, col));
                mma_bf16(sc[0], qf[kk], kf[0], kf[1]);
                mma_bf16(sc[1], qf[kk], kf[2], kf[3]);
            }
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int rr = e >> 1;
                    const int64_t tj = ts[kw + nt * 8 + 2 * t4 + (e & 1)];
                    const int64_t ti = t_row[rr];
                    const bool vis = ti >= 0 && tj >= 0 && tj <= ti && (a.window <= 0 || tj > ti - a.window);
                    // The reference stores q.k in bf16 before scaling (gpt_oss.py:133-151 in a bf16 graph).
                    sc[nt][e] = vis ? bf16_round(sc[nt][e]) : -INFINITY;
                    mx[rr] = fmaxf(mx[rr], sc[nt][e]);
                }
            }
            float corr[2], neg[2], rs[2] = {0.f, 0.f};
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 1));
                mx[rr] = fmaxf(mx[rr], __shfl_xor_sync(0xffffffffu, mx[rr], 2));
                const float m_new = fmaxf(m_run[rr], mx[rr] * a.scale_log2);
                const bool none = m_new == -INFINITY;
                corr[rr] = none ? 1.f : fast_exp2(m_run[rr] - m_new);
                neg[rr] = none ? 0.f : -m_new;
                m_run[rr] = m_new;
            }
            uint32_t af[4];
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                float pv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    pv[e] = fast_exp2(fmaf(sc[nt][e], a.scale_log2, neg[e >> 1]));
                    rs[e >> 1] += pv[e];
                }
                af[nt * 2 + 0] = pack_bf16(pv[0], pv[1]);
                af[nt * 2 + 1] = pack_bf16(pv[2], pv[3]);
            }
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) l_run[rr] = l_run[rr] * corr[rr] + rs[rr];
#pragma unroll
            for (int nd = 0; nd < 8; ++nd) {
                o[nd][0] *= corr[0];
                o[nd][1] *= corr[0];
                o[nd][2] *= corr[1];
                o[nd][3] *= corr[1];
            }
#pragma unroll
            for (int nd = 0; nd < 8; nd += 2) {
                uint32_t vf[4];
                const int key = kw + (lane & 7) + 8 * ((lane >> 3) & 1);
                const int col = nd * 8 + 8 * (lane >> 4);
                ldsm_x4_t(vf, Vb + fa_swz(key, col));
                mma_bf16(o[nd], af, vf[0], vf[1]);
                mma_bf16(o[nd + 1], af, vf[2], vf[3]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
        }
    }

    __syncthreads();  // every tile consumed: the ring is free for the merge

    // Merge the 4 consumer warps (shared memory reused: [warp][16 rows][64] outputs, then max and sum per warp and row).
    float* wo = reinterpret_cast<float*>(ring);  // 4 x 16 x 64 floats = 16 KB
    float* wm = wo + 4 * kFdRows * kFaDim;      // 4 x 16
    float* wl = wm + 4 * kFdRows;               // 4 x 16
    if (warp < 4) {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 1);
            l_run[rr] += __shfl_xor_sync(0xffffffffu, l_run[rr], 2);
        }
#pragma unroll
        for (int nd = 0; nd < 8; ++nd) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int r = g + 8 * (e >> 1), c = nd * 8 + 2 * t4 + (e & 1);
                wo[(warp * kFdRows + r) * kFaDim + c] = o[nd][e];
            }
        }
        if (t4 == 0) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr) {
                wm[warp * kFdRows + g + 8 * rr] = m_run[rr];
                wl[warp * kFdRows + g + 8 * rr] = l_run[rr];
            }
        }
    }
    __syncthreads();
    float* pp = a.part + ((size_t(b) * a.KV + kvh) * a.splits + split) * kFdRows * (2 + kFaDim);
    if (threadIdx.x < 128) {  // thread -> (row, 8 columns): 16 rows x 8 column groups
        const int r = threadIdx.x >> 3, c0 = (threadIdx.x & 7) * 8;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w * kFdRows + r]);
        float L = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float mw = wm[w * kFdRows + r];
            const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - M);
            L += wl[w * kFdRows + r] * f;
#pragma unroll
            for (int c = 0; c < 8; ++c) acc[c] += wo[(w * kFdRows + r) * kFaDim + c0 + c] * f;
        }
        if (c0 == 0) {
            pp[r * (2 + kFaDim) + 0] = M;
            pp[r * (2 + kFaDim) + 1] = L;
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) pp[r * (2 + kFaDim) + 2 + c0 + c] = acc[c];
    }
    // The last split CTA of this (sequence, KV head) merges the splits with the sink.
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned* counter = a.counters + size_t(b) * a.KV + kvh;
        const unsigned prev = atomicAdd(counter, 1u);
        s_last = prev == unsigned(a.splits - 1);
        if (s_last) *counter = 0u;
    }
    __syncthreads();
    if (!s_last || threadIdx.x >= 128) return;
    __threadfence();
    const float* base = a.part + (size_t(b) * a.KV + kvh) * a.splits * kFdRows * (2 + kFaDim);
    const int r = threadIdx.x >> 3, c0 = (threadIdx.x & 7) * 8;
    if (r >= rows) return;
    float M = -INFINITY;
    for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, __ldcg(base + (size_t(sp) * kFdRows + r) * (2 + kFaDim)));
    const int h = kvh * a.G + r % a.G, i = r / a.G;
    const float sink = __bfloat162float(sinks[h]) * 1.4426950408889634f;
    const float mf = fmaxf(M, sink);
    float L = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int sp = 0; sp < a.splits; ++sp) {
        const float* row = base + (size_t(sp) * kFdRows + r) * (2 + kFaDim);
        const float ms = __ldcg(row);
        const float f = ms == -INFINITY ? 0.f : exp2f(ms - mf);
        L += __ldcg(row + 1) * f;
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] += __ldcg(row + 2 + c0 + c) * f;
    }
    const float inv = 1.0f / (L + exp2f(sink - mf));
    __nv_bfloat16* orow = out + ((size_t(b) * a.n + i) * a.H + h) * kFaDim + c0;
    *reinterpret_cast<uint4*>(orow) = make_uint4(pack_bf16(acc[0] * inv, acc[1] * inv), pack_bf16(acc[2] * inv, acc[3] * inv),
                                                 pack_bf16(acc[4] * inv, acc[5] * inv), pack_bf16(acc[6] * inv, acc[7] * inv));
}

}  // namespace cb200
