// Test program (compiled by tests/test_gpu_sigmoid.py): the shipped fast_sigmoid_bf16in against
// bf16(1.0f / (1.0f + expf(-z))) for every one of the 65,536 bf16 inputs z, NaNs included. Prints the count of
// inputs whose bf16 results differ, then those inputs.
#include <cstdio>
#include <cstring>

#include "common.cuh"

__global__ void k_check(unsigned* count, unsigned short* which) {
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= 65536u) return;
    const float z = __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(i)));
    const unsigned short want = __bfloat16_as_ushort(__float2bfloat16_rn(1.0f / (1.0f + expf(-z))));
    const unsigned short got = __bfloat16_as_ushort(__float2bfloat16_rn(cb200::fast_sigmoid_bf16in(z)));
    if (want != got) {
        const unsigned slot = atomicAdd(count, 1u);
        if (slot < 64) which[slot] = static_cast<unsigned short>(i);
    }
}

int main() {
    unsigned* count = nullptr;
    unsigned short* which = nullptr;
    if (cudaMalloc(&count, 4) != cudaSuccess || cudaMalloc(&which, 128) != cudaSuccess) return 2;
    cudaMemset(count, 0, 4);
    k_check<<<256, 256>>>(count, which);
    unsigned h = 0;
    unsigned short hw[64];
    if (cudaMemcpy(&h, count, 4, cudaMemcpyDeviceToHost) != cudaSuccess) return 3;
    cudaMemcpy(hw, which, sizeof(hw), cudaMemcpyDeviceToHost);
    printf("%u\n", h);
    for (unsigned i = 0; i < h && i < 64; ++i) printf("0x%04x\n", hw[i]);
    return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
