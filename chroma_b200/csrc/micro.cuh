// Fused RMSNorm + gated SiLU + residual over bf16 rows (the C3 micrograph):
//   y = bf16(x * (1/sqrt(mean(x^2) + eps)) * w)      fused fp32 norm, rounded once (kernels.h:101-115)
//   z = bf16(y * g); s = bf16(sigmoid(z)); out = bf16(bf16(bf16(z * s) * u) + x)
// with the reference's rounding after every exported bf16 op (chroma/_src/lowering.py:185-210). One CTA per row,
// 16-byte vector loads of 8 bf16; the x row stays in registers between the reduction and the epilogue, and g/u are
// requested before the reduction completes so their DRAM latency overlaps it. HBM traffic is the algorithmic
// minimum: 3 reads + 1 write of each element plus the norm weight (L2-resident).
#pragma once

#include "common.cuh"

namespace cb200 {

// Rows of up to 2 chunks per thread (C3: 4,096 columns, 256 threads) are held to 40 registers, so six CTAs fit an
// SM instead of four: 87 us instead of 103 us at C3, the loads of more rows in flight.
template <int CHUNKS>
__global__ void __launch_bounds__(512, CHUNKS <= 2 ? 3 : 1) k_micro(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ g,
                                                const __nv_bfloat16* __restrict__ u, const float* __restrict__ w,
                                                __nv_bfloat16* __restrict__ out, int64_t rows, int cols, float eps) {
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5, warps = blockDim.x >> 5;
    const int per_chunk = blockDim.x * 8;  // elements covered by one chunk of all threads
    const size_t base = size_t(row) * cols;
    pdl_wait();
    pdl_trigger();

    uint4 xv[CHUNKS], gv[CHUNKS], uv[CHUNKS];
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = c * per_chunk + tid * 8;
        if (col < cols) xv[c] = __ldcs(reinterpret_cast<const uint4*>(x + base + col));
    }
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = c * per_chunk + tid * 8;
        if (col < cols) {
            gv[c] = __ldcs(reinterpret_cast<const uint4*>(g + base + col));
            uv[c] = __ldcs(reinterpret_cast<const uint4*>(u + base + col));
        }
    }
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = c * per_chunk + tid * 8;
        if (col < cols) {
            const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&xv[c]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __bfloat1622float2(p[i]);
                s = fmaf(f.x, f.x, s);
                s = fmaf(f.y, f.y, s);
            }
        }
    }
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (warp == 0) {
        float t = lane < warps ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[0] = 1.0f / sqrtf(t / float(cols) + eps);
    }
    __syncthreads();
    const float inv = red[0];
#pragma unroll
    for (int c = 0; c < CHUNKS; ++c) {
        const int col = c * per_chunk + tid * 8;
        if (col >= cols) continue;
        const __nv_bfloat162* px = reinterpret_cast<const __nv_bfloat162*>(&xv[c]);
        const __nv_bfloat162* pg = reinterpret_cast<const __nv_bfloat162*>(&gv[c]);
        const __nv_bfloat162* pu = reinterpret_cast<const __nv_bfloat162*>(&uv[c]);
        const float4 w0 = *reinterpret_cast<const float4*>(w + col);
        const float4 w1 = *reinterpret_cast<const float4*>(w + col + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint4 ov;
        __nv_bfloat162* po = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            // Two elements at a time. A product of two bf16 values is exact in fp32, so the packed bf16
            // multiplies (one rounding of the exact product) give the bits of "fp32 multiply, round to bf16".
            const float2 fx = __bfloat1622float2(px[i]);
            const __nv_bfloat162 y = __floats2bfloat162_rn(__fmul_rn(__fmul_rn(fx.x, inv), wv[2 * i]),
                                                           __fmul_rn(__fmul_rn(fx.y, inv), wv[2 * i + 1]));
            const __nv_bfloat162 z = __hmul2(y, pg[i]);
            const float2 fz = __bfloat1622float2(z);
            const __nv_bfloat162 sg = __floats2bfloat162_rn(fast_sigmoid_bf16in(fz.x), fast_sigmoid_bf16in(fz.y));
            const float2 fb = __bfloat1622float2(__hmul2(__hmul2(z, sg), pu[i]));
            po[i] = __floats2bfloat162_rn(__fadd_rn(fb.x, fx.x), __fadd_rn(fb.y, fx.y));
        }
        __stcs(reinterpret_cast<uint4*>(out + base + col), ov);
    }
}

}  // namespace cb200
