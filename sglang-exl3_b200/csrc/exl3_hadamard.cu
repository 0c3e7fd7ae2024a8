// Stand-alone input rotation: out = fp16 H128(x * suh) / sqrt(128) per 128-block
// of each row.  Replaces the upstream exllamav3 had_r_128 that the reference's
// fat-GEMM MoE path calls before exl3_fat_gemm (src/sglang_exl3/exl3.py:1184-1193).
#include "exl3_common.cuh"
#include "exl3_capi_internal.h"

namespace exl3b200 {

__global__ __launch_bounds__(256) void exl3_hadamard_in_kernel(const __half* __restrict__ x, long long x_stride,
                                                               const __half* __restrict__ suh, __half* __restrict__ out,
                                                               long long out_stride, int m, int k)
{
    const int lane = threadIdx.x & 31;
    const int nblk = k >> 7;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < m * nblk; task += warps) {
        const int row = task / nblk;
        const int b = task - row * nblk;
        __half h[4];
        rotate_block(x + (size_t) row * x_stride + b * 128, suh ? suh + b * 128 : nullptr, lane, h);
#pragma unroll
        for (int i = 0; i < 4; ++i) out[(size_t) row * out_stride + b * 128 + lane + 32 * i] = h[i];
    }
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" int exl3b200_hadamard_in(const void* x, long long x_stride, int m, int k, const void* suh, void* out,
                                    long long out_stride, void* stream)
{
    if (!x || !out) return kErrNullPointer;
    if (m < 1 || k <= 0 || (k % 128) || x_stride < k || out_stride < k) return kErrBadShape;
    if (((uintptr_t) x & 1) || ((uintptr_t) out & 1)) return kErrUnaligned;
    const int tasks = m * (k / 128);
    const int grid = std::min((tasks + 7) / 8, 8 * 148);
    exl3_hadamard_in_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const __half*>(x), x_stride, reinterpret_cast<const __half*>(suh),
        reinterpret_cast<__half*>(out), out_stride, m, k);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}
