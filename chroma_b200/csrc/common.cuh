// Shared device helpers for the B200 (sm_100a) kernels of chroma_b200.
//
// Numerics follow the reference's storage rules: every kernel computes in fp32; a value the reference keeps
// in bf16 is rounded to nearest-even at the same points (chroma/_src/core/bfloat16.h:7-17,
// chroma/_src/codegen/cuda/codegen.py:62-66 uses __float2bfloat16_rn for the same purpose).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cb200 {

// Error bits written by kernels into the per-program error word (the role of the index-error flag at
// chroma/_src/codegen/cuda/runtime.h:18-32).
enum : unsigned int { kErrIndex = 1u, kErrTimeout = 2u };

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// sigmoid(z) = 1 / (1 + exp(-z)) for a z that is a bf16 value, on the special-function unit: __expf and the
// approximate reciprocal (rcp.approx.f32, full range) instead of expf and the correctly rounded division (the C3
// micrograph was issue-bound on those two sequences). The result is only ever rounded to bf16, and for every one of
// the 65,536 bf16 inputs (NaNs included) this form gives the same bf16 bits as bf16(1.0f / (1.0f + expf(-z))) on
// the B200, checked exhaustively (__fdividef(1, .) in its place differs on z = -87.5, -88, -88.5, where the divisor
// exceeds 2^126 and it returns 0).
__device__ __forceinline__ float fast_sigmoid_bf16in(float z) {
    const float den = __fadd_rn(1.0f, __expf(-z));
    float r;
    asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(den));
    return r;
}

// Storage precision policy: Round<float> is the identity, Round<bf16> rounds to bf16 and back.
template <typename T> struct Store;
template <> struct Store<float> {
    static __device__ __forceinline__ float round(float x) { return x; }
    static __device__ __forceinline__ float load(const float* p) { return *p; }
    static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
    static constexpr bool bf16 = false;
};
template <> struct Store<__nv_bfloat16> {
    static __device__ __forceinline__ float round(float x) { return bf16_round(x); }
    static __device__ __forceinline__ float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
    static __device__ __forceinline__ void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
    static constexpr bool bf16 = true;
};

// Loads four consecutive storage elements (16 B for fp32, 8 B for bf16) as floats. The pointer must be
// aligned to the access size; every caller indexes rows whose length is a multiple of 4.
__device__ __forceinline__ void load4(const float* p, float (&v)[4]) {
    float4 q = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
__device__ __forceinline__ void load4(const __nv_bfloat16* p, float (&v)[4]) {
    uint2 q = __ldg(reinterpret_cast<const uint2*>(p));
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&q.x);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&q.y);
    float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
    v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
}
// Streaming variant for weights read exactly once per launch: bypass L1 allocation. Not volatile, so the
// compiler may batch several of these ahead of their uses (the data is read-only for the kernel's lifetime).
__device__ __forceinline__ void load4_stream(const float* p, float (&v)[4]) {
    float4 q;
    asm("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(q.x), "=f"(q.y), "=f"(q.z), "=f"(q.w) : "l"(p));
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
}
__device__ __forceinline__ void load4_stream(const __nv_bfloat16* p, float (&v)[4]) {
    uint32_t a, b;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(a), "=r"(b) : "l"(p));
    __nv_bfloat162 pa = *reinterpret_cast<__nv_bfloat162*>(&a);
    __nv_bfloat162 pb = *reinterpret_cast<__nv_bfloat162*>(&b);
    float2 fa = __bfloat1622float2(pa), fb = __bfloat1622float2(pb);
    v[0] = fa.x; v[1] = fa.y; v[2] = fb.x; v[3] = fb.y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
// Sum within aligned groups of `width` lanes (width a power of two <= 32).
__device__ __forceinline__ float group_sum(float v, int width) {
    for (int o = width >> 1; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Bounds-checked row index with optional negative wrap-around (aten.index semantics), the device-side
// counterpart of chroma::cuda::index (chroma/_src/codegen/cuda/runtime.h:18-32). An invalid value raises
// the index bit and reads row 0 so the kernel can finish; the host turns the bit into IndexError.
__device__ __forceinline__ int64_t checked_row(int64_t value, int64_t count, bool negative, unsigned int* error) {
    if (value >= 0 && value < count) return value;
    if (negative && value < 0 && value >= -count) return value + count;
    atomicOr(error, kErrIndex);
    return 0;
}

// Programmatic dependent launch (Hopper+): a kernel may start while its predecessor drains. Everything
// before pdl_wait() must touch only data no earlier kernel writes (weights); pdl_trigger() lets the next
// kernel in the stream begin launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// L2 prefetch of a byte range (weights a CTA will read after pdl_wait()).
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes, int lane, int lanes) {
    const char* c = static_cast<const char*>(p);
    for (size_t off = size_t(lane) * 128; off < bytes; off += size_t(lanes) * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(c + off));
}

// Grid-stride L2 prefetch of a byte range (one 128-byte line per thread step).
__global__ void k_prefetch_l2(const char* base, size_t bytes) {
    const size_t lines = (bytes + 127) / 128;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < lines; i += size_t(gridDim.x) * blockDim.x)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(base + i * 128));
}

// L2 prefetch of `bytes` (a multiple of 16) at 16-byte aligned `p` by the TMA engine: one instruction, no data
// returned to the SM.
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Grid-stride bulk L2 prefetch of a 16-byte aligned range in 64 KiB pieces (one thread per piece).
__global__ void k_prefetch_l2_bulk(const char* base, size_t bytes) {
    constexpr size_t kPiece = 64 * 1024;
    const size_t pieces = (bytes + kPiece - 1) / kPiece;
    for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < pieces; i += size_t(gridDim.x) * blockDim.x) {
        const size_t off = i * kPiece;
        const size_t n = bytes - off < kPiece ? bytes - off : kPiece;
        bulk_prefetch_l2(base + off, unsigned(n & ~size_t(15)));
    }
}

// Orderable 64-bit argmax key: larger value wins, then the lower index (numpy.argmax: first occurrence).
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
    unsigned u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    if (isnan(v)) u = 0xffffffffu;
    return (static_cast<unsigned long long>(u) << 32) | (0xffffffffu - static_cast<unsigned>(idx));
}

__host__ __device__ inline int64_t argmax_index(unsigned long long key) {
    return int64_t(0xffffffffu - static_cast<unsigned>(key & 0xffffffffull));
}

}  // namespace cb200
