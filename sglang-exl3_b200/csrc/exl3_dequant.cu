// Trellis -> fp16 weight reconstruction ("dequant_trellis"), bit-exact.
//
// Replaces the reference's single-threaded CPU dequant_cpu
// (csrc/bindings.cpp:15-100) with one CTA per 128x128 Hadamard block:
//   1. each warp decodes whole 16x16 tiles (windows + codebook) straight into a
//      float32 block in shared memory, at the fragment-swizzled positions;
//   2. one warp per row runs the 128-point transform over columns, * 1/sqrt(128);
//   3. one warp per column runs it over rows, then * 1/sqrt(128) * suh[k] * svh[n],
//      and the block is stored row-major with one fp16 rounding.
// Every float operation is an explicit round-to-nearest intrinsic in the order
// of the reference loop, so the output is bit-identical to it.  Codebook
// rounding is selectable: round-to-nearest (the semantics of the reference's
// device decode, csrc/quant/codebook.cuh) or truncation (the semantics of the
// reference's CPU helpers, csrc/exl3_dequant.cuh:41-93, i.e. of its
// dequant_trellis op).
#include "exl3_common.cuh"
#include "exl3_capi_internal.h"

namespace exl3b200 {

constexpr int kDqThreads = 256;
constexpr int kDqStride = 129;  // padded row stride of the float block (bank-conflict free both ways)

template <int K, int CB, bool TRUNC>
__global__ __launch_bounds__(kDqThreads) void dequant_kernel(
    const uint16_t* __restrict__ trellis, const __half* __restrict__ suh, const __half* __restrict__ svh,
    __half* __restrict__ out, int k_tiles, int n_tiles)
{
    extern __shared__ float smem[];
    float* blk = smem;                                   // [128][129]
    uint32_t* wbuf = reinterpret_cast<uint32_t*>(smem + 128 * kDqStride);  // [8 warps][8K words]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int nb = blockIdx.x;  // 128-column block
    const int kb = blockIdx.y;  // 128-row block
    const int n_cols = n_tiles * 16;
    constexpr int TW = 8 * K;  // uint32 words per tile

    uint32_t* my_words = wbuf + warp * TW;

    // 1. decode the 64 tiles of the block (8 per warp)
    for (int tt = warp; tt < 64; tt += kDqThreads / 32) {
        const int kt = kb * 8 + (tt >> 3);
        const int nt = nb * 8 + (tt & 7);
        const uint32_t* src = reinterpret_cast<const uint32_t*>(trellis + ((size_t) kt * n_tiles + nt) * 16 * K);
        for (int i = lane; i < TW; i += 32) my_words[i] = src[i];
        __syncwarp();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int t = lane * 8 + j;
            const uint32_t w = tile_window<K>(my_words, t);
            const float v = TRUNC ? codebook_value_trunc<CB>(w) : codebook_value_rn<CB>(w);
            const int k = 2 * (lane & 3) + (j & 1) + 8 * ((j >> 1) & 1);
            const int n = (lane >> 2) + 8 * (j >> 2);
            blk[((tt >> 3) * 16 + k) * kDqStride + (tt & 7) * 16 + n] = v;
        }
        __syncwarp();
    }
    __syncthreads();

    // 2. transform every row over its 128 columns
    for (int r = warp; r < 128; r += kDqThreads / 32) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = blk[r * kDqStride + lane + 32 * i];
        warp_fwht128(v, lane);
#pragma unroll
        for (int i = 0; i < 4; ++i) blk[r * kDqStride + lane + 32 * i] = __fmul_rn(v[i], kHadScale);
    }
    __syncthreads();

    // 3. transform every column over its 128 rows, scale, keep in the block
    for (int c = warp; c < 128; c += kDqThreads / 32) {
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = blk[(lane + 32 * i) * kDqStride + c];
        warp_fwht128(v, lane);
        const float sv = __half2float(svh[nb * 128 + c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float su = __half2float(suh[kb * 128 + lane + 32 * i]);
            blk[(lane + 32 * i) * kDqStride + c] = __fmul_rn(__fmul_rn(__fmul_rn(v[i], kHadScale), su), sv);
        }
    }
    __syncthreads();

    // 4. coalesced fp16 store of the block
    for (int idx = threadIdx.x; idx < 128 * 64; idx += kDqThreads) {
        const int r = idx >> 6;
        const int c2 = (idx & 63) * 2;
        const __half2 h = __floats2half2_rn(blk[r * kDqStride + c2], blk[r * kDqStride + c2 + 1]);
        *reinterpret_cast<__half2*>(out + (size_t) (kb * 128 + r) * n_cols + nb * 128 + c2) = h;
    }
}

template <int K, int CB, bool TRUNC>
static int launch_dequant(const uint16_t* trellis, const __half* suh, const __half* svh, __half* out,
                          int k_tiles, int n_tiles, cudaStream_t stream)
{
    const size_t smem = (size_t) 128 * kDqStride * sizeof(float) + (size_t) 8 * 8 * K * sizeof(uint32_t);
    auto kern = dequant_kernel<K, CB, TRUNC>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) != cudaSuccess)
        return kErrLaunch;
    dim3 grid(n_tiles / 8, k_tiles / 8);
    kern<<<grid, kDqThreads, smem, stream>>>(trellis, suh, svh, out, k_tiles, n_tiles);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

template <int K>
static int dispatch_cb(int cb, bool trunc, const uint16_t* trellis, const __half* suh, const __half* svh,
                       __half* out, int k_tiles, int n_tiles, cudaStream_t stream)
{
    if (trunc) {
        if (cb == 0) return launch_dequant<K, 0, true>(trellis, suh, svh, out, k_tiles, n_tiles, stream);
        if (cb == 1) return launch_dequant<K, 1, true>(trellis, suh, svh, out, k_tiles, n_tiles, stream);
        return launch_dequant<K, 2, true>(trellis, suh, svh, out, k_tiles, n_tiles, stream);
    }
    if (cb == 0) return launch_dequant<K, 0, false>(trellis, suh, svh, out, k_tiles, n_tiles, stream);
    if (cb == 1) return launch_dequant<K, 1, false>(trellis, suh, svh, out, k_tiles, n_tiles, stream);
    return launch_dequant<K, 2, false>(trellis, suh, svh, out, k_tiles, n_tiles, stream);
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" int exl3b200_dequant(const void* trellis, int k_tiles, int n_tiles, int K, int cb,
                                const void* suh, const void* svh, void* out, int rounding, void* stream)
{
    if (!trellis || !suh || !svh || !out) return kErrNullPointer;
    if (K < 1 || K > 8) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (rounding != 0 && rounding != 1) return kErrBadArgument;
    if (k_tiles <= 0 || n_tiles <= 0 || (k_tiles % 8) || (n_tiles % 8)) return kErrBadShape;
    if (((uintptr_t) trellis & 3) || ((uintptr_t) out & 3)) return kErrUnaligned;
    const bool trunc = rounding == 1;
    auto tr = reinterpret_cast<const uint16_t*>(trellis);
    auto su = reinterpret_cast<const __half*>(suh);
    auto sv = reinterpret_cast<const __half*>(svh);
    auto o = reinterpret_cast<__half*>(out);
    auto st = reinterpret_cast<cudaStream_t>(stream);
    switch (K) {
        case 1: return dispatch_cb<1>(cb, trunc, tr, su, sv, o, k_tiles, n_tiles, st);
        case 2: return dispatch_cb<2>(cb, trunc, tr, su, sv, o, k_tiles, n_tiles, st);
        case 3: return dispatch_cb<3>(cb, trunc, tr, su, sv, o, k_tiles, n_tiles, st);
        case 4: return dispatch_cb<4>(cb, trunc, tr, su, sv, o, k_tiles, n_tiles, st);
        case 5: return dispatch_cb<5>(cb, trunc, tr, su, sv, o, k_tiles, n_tiles, st);
        case 6: return dispatch_cb<6>(cb, trunc, tr, su, sv, o, k_tiles, n_tiles, st);
        case 7: return dispatch_cb<7>(cb, trunc, tr, su, sv, o, k_tiles, n_tiles, st);
        default: return dispatch_cb<8>(cb, trunc, tr, su, sv, o, k_tiles, n_tiles, st);
    }
}
