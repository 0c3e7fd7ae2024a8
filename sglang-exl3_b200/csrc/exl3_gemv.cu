// Small-M EXL3 matmul (M <= 16 rows): y = H128(H128(x * suh) @ W_raw) * svh / 128.
//
// Replaces the reference's cooperative QTIP-style GEMV
// (csrc/quant/exl3_gemv_kernel.cuh:138-402, host csrc/exl3_gemv.cu:26-63) with a
// design for B200:
//
// * input stage (exl3_input_kernel): one warp per (row, 128-block) computes the
//   fp16 x_had = H128(x * suh) / sqrt(128) with the reference's roundings
//   (had_hf_r_128_inner<true,false>, csrc/quant/hadamard_inner.cuh:93-147) into
//   the caller's workspace.  The matmul kernel is launched as its programmatic
//   dependent (PDL), so its trellis loads start while the input stage runs and
//   only the x_had reads wait (griddepcontrol.wait).  No grid-wide barrier.
// * matmul (exl3_gemv_kernel): the iteration space is the list of units
//   (128-column block nb, 16-row k-slice kr), nb-major; the grid (2 CTAs per
//   SM) splits it evenly ("stream-K"), so any shape load-balances over 148 SMs.
//   Each warp of a CTA takes k-slices of the current block and, per slice,
//   streams the block's 8 tiles with coalesced 32-bit loads (one 128-byte
//   transaction per tile at 4 bpw) through a register ring a few slices deep,
//   resolves each lane's two stream words with one or two shuffles, extracts the
//   8 windows and runs the codebook in registers.  The decoded 16x16 tile is
//   used transposed as the A operand of mma.m16n8k16 (rows = output columns,
//   cols = k) and x_had as B (k x 8 tokens), fp32 accumulate, so at M <= 8 no
//   tensor work is spent on padding rows.  The codebook's final fp16 add
//   (cb 0/1) is folded into the MMA: the LOP3 word {lo, hi} goes in as a k pair
//   against a duplicated activation {h, h} (written so by the input stage),
//   which saves the PRMT/HADD2 of every weight pair for one extra MMA per tile;
//   the integer-logic pipe (half rate on sm_100) is what bounds this kernel, so
//   window extraction uses byte permutes and FMA-pipe shifts where it can.
//   mul1 (cb 2) feeds the exact
//   integer-valued fp16 h = 1024 + bytesum and applies
//   y = k_inv * sum(x h) + k_bias * sum(x) in float in the epilogue.
// * reduction: warps add their fragments into a shared [rows][128] block; a CTA
//   that covered all k-slices of the block runs the epilogue itself, otherwise it
//   adds the block into an fp32 workspace slice and the last of the block's
//   contributors (an atomic arrival counter, no waiting) runs the epilogue and
//   re-zeroes the slice and counter for the next call.
// * epilogue: one warp per row: H128 over the 128 columns, * 1/sqrt(128) * svh,
//   one rounding to the output dtype (fp16 / bf16 / fp32), strided store.
#include "exl3_common.cuh"
#include "exl3_capi_internal.h"

namespace exl3b200 {

constexpr int kGvThreads = 256;
constexpr int kGvWarps = kGvThreads / 32;
constexpr int kRedStride = 132;  // padded row stride of the shared reduction block

struct GemvParams {
    const uint32_t* xd;      // [M, k] rotated input as duplicated fp16 pairs {h, h}
    const uint32_t* trellis; // [k/16, n/16, 16K] as uint32 words
    const __half* svh;       // [n]
    const float* sblk;       // [M, k/128] block sums of xh (cb 2 only)
    void* out;               // [M, out_stride]
    float* ws_acc;           // [n/128, 16, 128] zeroed fp32 partial sums
    long long out_stride;
    int out_dtype;
    int m;
    int k;
    int n;
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// input stage
// ---------------------------------------------------------------------------

// One warp per (row, 128-block): h = fp16(H128(fp16(x * suh)) / sqrt(128)).
// Writes h to xh (if non-null, fp16 [m][xh_stride]) and/or the duplicated pairs
// {h, h} to xd (if non-null, uint32 [m][k]) - the B fragments of the folded MMA.
__global__ __launch_bounds__(256) void exl3_input_kernel(
    const __half* __restrict__ x, long long x_stride, const __half* __restrict__ suh,
    __half* __restrict__ xh, long long xh_stride, uint32_t* __restrict__ xd, float* __restrict__ sblk,
    int m, int k, int rotate)
{
    griddep_launch();
    const int lane = threadIdx.x & 31;
    const int nblk = k >> 7;
    const int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (task >= m * nblk) return;
    const int row = task / nblk;
    const int b = task - row * nblk;
    const __half* src = x + row * x_stride + b * 128;
    float v[4];
    __half h[4];
    if (rotate) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float xv = __half2float(src[lane + 32 * i]);
            v[i] = suh ? __half2float(__float2half_rn(__fmul_rn(xv, __half2float(suh[b * 128 + lane + 32 * i]))))
                       : xv;
        }
        warp_fwht128(v, lane);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __float2half_rn(__fmul_rn(v[i], kHadScale));
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = src[lane + 32 * i];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const size_t col = (size_t) b * 128 + lane + 32 * i;
        if (xh) xh[(size_t) row * xh_stride + col] = h[i];
        if (xd) {
            const uint32_t u = __half_as_ushort(h[i]);
            xd[(size_t) row * k + col] = u | (u << 16);
        }
        v[i] = __half2float(h[i]);
    }
    if (sblk) {
        float s = (v[0] + v[1]) + (v[2] + v[3]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sblk[(size_t) row * nblk + b] = s;
    }
}

// ---------------------------------------------------------------------------
// matmul
// ---------------------------------------------------------------------------

// Loads per k-slice per lane for the 8 tiles of a block: tiles are 8K words;
// K = 1, 2, 4 pack 32/(8K) tiles into one 32-lane load, K = 3 loads one tile per
// load on 24 lanes.
template <int K, int NT>
struct SliceLoad {
    static constexpr int TW = 8 * K;
    static constexpr int LOADS = (K == 3) ? NT : (NT * TW) / 32;
};

// K bits, codebook CB, TG groups of 8 rows, NT tiles per warp per k-slice (8 or 4:
// with 4, two warps share a slice's 8-tile block), P-deep trellis register ring.
template <int K, int CB, int TG, int NT, int P, int MINB>
__global__ __launch_bounds__(kGvThreads, MINB) void exl3_gemv_kernel(const GemvParams p)
{
    griddep_launch();  // let the epilogue kernel get scheduled early; it waits for this grid
    constexpr int TW = SliceLoad<K, NT>::TW;
    constexpr int LOADS = SliceLoad<K, NT>::LOADS;
    constexpr int TGRP = 8 / NT;            // warps sharing one slice
    constexpr int SG = kGvWarps / TGRP;     // slice groups

    __shared__ float red[TG * 8][kRedStride];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int c = lane & 3;
    const LaneWords lw = lane_words<K>(lane);

    const int kt_total = p.k >> 4;
    const int n_tiles = p.n >> 4;
    const int nblocks = p.n >> 7;
    const long long units = (long long) nblocks * kt_total;
    const long long G = gridDim.x;
    const long long u_begin = (long long) blockIdx.x * units / G;
    const long long u_end = (long long) (blockIdx.x + 1) * units / G;

    // K = 3: 24 of 32 lanes carry a tile's words
    const bool load_lane = (K != 3) || lane < 24;
    const size_t slice_words = (size_t) n_tiles * TW;  // words per k-slice row of the matrix

    bool waited = false;

    for (long long u = u_begin; u < u_end;) {
        const int nb = (int) (u / kt_total);
        const int kr0 = (int) (u - (long long) nb * kt_total);
        const int len = (int) min((long long) (kt_total - kr0), u_end - u);

        for (int i = threadIdx.x; i < TG * 8 * kRedStride; i += kGvThreads) (&red[0][0])[i] = 0.f;

        float acc[NT][TG][4];
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int q = 0; q < TG; ++q)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[t][q][r] = 0.f;

        // this warp's tiles th*NT.. and slices kr0 + sg + SG * i, i < nr
        const int th = warp % TGRP;
        const int sg = warp / TGRP;
        const int nr = len > sg ? (len - sg + SG - 1) / SG : 0;
        const uint32_t* bptr =
            p.trellis + (size_t) (kr0 + sg) * slice_words + (size_t) (nb * 8 + th * NT) * TW + lane;
        const size_t bstep = slice_words * SG;
        // activation fragments: row 8q + g, k = kr*16 + 2c (+8), as {h,h} pairs
        const uint2* xptr[TG];
        bool xrow[TG];
#pragma unroll
        for (int q = 0; q < TG; ++q) {
            const int row = 8 * q + g;
            xrow[q] = row < p.m;
            xptr[q] = reinterpret_cast<const uint2*>(p.xd + (size_t) (xrow[q] ? row : 0) * p.k +
                                                     (size_t) (kr0 + sg) * 16 + 2 * c);
        }
        const size_t xstep = (size_t) SG * 16 / 2;  // in uint2

        uint32_t ring[P][LOADS];
        uint2 xnext[TG][2];
        auto load_slice = [&](int i, uint32_t (&dst)[LOADS]) {
            const uint32_t* bp = bptr + (size_t) i * bstep;
#pragma unroll
            for (int l = 0; l < LOADS; ++l) {
                const int off = (K == 3) ? l * TW : l * 32;
                dst[l] = load_lane ? __ldcs(bp + off) : 0u;
            }
        };
        auto load_x = [&](int i, uint2 (&dst)[TG][2]) {
#pragma unroll
            for (int q = 0; q < TG; ++q) {
                if (xrow[q]) {
                    const uint2* xp = xptr[q] + (size_t) i * xstep;
                    dst[q][0] = __ldcg(xp);
                    dst[q][1] = __ldcg(xp + 4);
                } else {
                    dst[q][0] = make_uint2(0u, 0u);
                    dst[q][1] = make_uint2(0u, 0u);
                }
            }
        };
        auto consume = [&](const uint32_t (&bw)[LOADS], const uint2 (&xb)[TG][2]) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                uint32_t wa, wb;
                if constexpr (K == 4) {
                    wb = bw[t];
                    wa = __shfl_sync(0xffffffffu, bw[t], (lane + 31) & 31);
                } else if constexpr (K == 3) {
                    wa = __shfl_sync(0xffffffffu, bw[t], lw.wa);
                    wb = __shfl_sync(0xffffffffu, bw[t], lw.wb);
                } else {
                    constexpr int TPL = 32 / TW;  // tiles per load
                    const uint32_t src = bw[t / TPL];
                    const int base = (t % TPL) * TW;
                    wa = __shfl_sync(0xffffffffu, src, base + lw.wa);
                    wb = __shfl_sync(0xffffffffu, src, base + lw.wb);
                }
                uint32_t w[8];
                lane_windows<K>(wa, wb, lw.shift7, w);
                uint32_t pv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) pv[j] = codebook_pre<CB>(w[j]);
                // folded A fragments: weight j's {lo, hi} as a k pair
                const uint32_t aA[4] = {pv[0], pv[4], pv[1], pv[5]};  // k = 2c, 2c+1
                const uint32_t aB[4] = {pv[2], pv[6], pv[3], pv[7]};  // k = 2c+8, 2c+9
#pragma unroll
                for (int q = 0; q < TG; ++q) {
                    mma_16816(aA, xb[q][0].x, xb[q][0].y, acc[t][q]);
                    mma_16816(aB, xb[q][1].x, xb[q][1].y, acc[t][q]);
                }
            }
        };

#pragma unroll
        for (int s = 0; s < P; ++s)
            if (s < nr) load_slice(s, ring[s]);
        if (!waited) {
            griddep_wait();
            waited = true;
        }
        if (nr > 0) load_x(0, xnext);

        // activations run one slice ahead (L2 hits), trellis P slices ahead
        auto step = [&](int i, int s) {
            uint32_t bw[LOADS];
            uint2 xb[TG][2];
#pragma unroll
            for (int l = 0; l < LOADS; ++l) bw[l] = ring[s][l];
#pragma unroll
            for (int q = 0; q < TG; ++q) {
                xb[q][0] = xnext[q][0];
                xb[q][1] = xnext[q][1];
            }
            if (i + P < nr) load_slice(i + P, ring[s]);
            if (i + 1 < nr) load_x(i + 1, xnext);
            consume(bw, xb);
        };
        int i = 0;
        for (; i + P <= nr; i += P) {
#pragma unroll
            for (int s = 0; s < P; ++s) step(i + s, s);
        }
#pragma unroll
        for (int s = 0; s < P; ++s)
            if (i + s < nr) step(i + s, s);

        __syncthreads();  // red zeroed by all threads before any atomics

        // fragment -> shared block: lane holds (n = 16t + g (+8), rows 8q + 2c (+1))
#pragma unroll
        for (int q = 0; q < TG; ++q) {
            const int r0 = 8 * q + 2 * c;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int n0 = 16 * (th * NT + t) + g;
                if (r0 < p.m) {
                    atomicAdd(&red[r0][n0], acc[t][q][0]);
                    atomicAdd(&red[r0][n0 + 8], acc[t][q][2]);
                }
                if (r0 + 1 < p.m) {
                    atomicAdd(&red[r0 + 1][n0], acc[t][q][1]);
                    atomicAdd(&red[r0 + 1][n0 + 8], acc[t][q][3]);
                }
            }
        }
        __syncthreads();

        // fire-and-forget: add this CTA's partial block into the zeroed state; the
        // epilogue kernel (a programmatic dependent of this grid) finishes it
        float* wsb = p.ws_acc + (size_t) nb * 16 * 128;
        for (int e = threadIdx.x; e < p.m * 128; e += kGvThreads) {
            const int r = e >> 7, col = e & 127;
            atomicAdd(wsb + r * 128 + col, red[r][col]);
        }
        __syncthreads();
        u += len;
    }
    if (!waited) griddep_wait();
}

// ---------------------------------------------------------------------------
// epilogue: one warp per (128-column block, row): read the summed partials and
// re-zero them, H128 over the block, * 1/sqrt(128) * svh, one rounding, store.
// Launched as a programmatic dependent of the matmul grid.
// ---------------------------------------------------------------------------
template <int CB>
__global__ __launch_bounds__(256) void exl3_gemv_epilogue_kernel(
    float* __restrict__ ws_acc, const __half* __restrict__ svh, const float* __restrict__ sblk, void* out,
    long long out_stride, int out_dtype, int m, int k, int n)
{
    const int lane = threadIdx.x & 31;
    const int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int nblocks = n >> 7;
    griddep_wait();
    if (task >= nblocks * m) return;
    const int nb = task % nblocks;
    const int r = task / nblocks;
    float* src = ws_acc + ((size_t) nb * 16 + r) * 128;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        v[e] = __ldcg(src + lane + 32 * e);
        __stcg(src + lane + 32 * e, 0.f);
    }
    if constexpr (CB == 2) {
        const float k_inv = __half2float(__ushort_as_half(kMul1InvBits));
        const float k_bias = __half2float(__ushort_as_half(kMul1BiasBits));
        const int nblk = k >> 7;
        float sum = 0.f;
        for (int b = lane; b < nblk; b += 32) sum += __ldcg(sblk + (size_t) r * nblk + b);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = fmaf(k_inv, v[e], k_bias * sum);
    }
    warp_fwht128(v, lane);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int col = nb * 128 + lane + 32 * e;
        store_out(out, (size_t) r * out_stride + col, v[e] * kHadScale * __half2float(svh[col]), out_dtype);
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static int sm_count()
{
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

static inline size_t align256(size_t v) { return (v + 255) & ~(size_t) 255; }

// state: [n/128][16][128] fp32 partial sums; zero when allocated, left zero by
// every call (the epilogue kernel re-zeroes what the matmul kernel added).
static size_t gemv_state_bytes(int n)
{
    const size_t nblocks = (size_t) n / 128;
    return align256(nblocks * 16 * 128 * sizeof(float));
}

// scratch: [m][k] rotated input as duplicated fp16 pairs, then [m][k/128] fp32 block sums.
static size_t gemv_scratch_bytes(int m, int k)
{
    return align256((size_t) m * k * sizeof(uint32_t)) + align256((size_t) m * (k / 128) * sizeof(float));
}

// Tiling variants (the kernel-shape map picks one per call):
//   0: 8 tiles per warp, 2 CTAs/SM    1: 4 tiles per warp, 3 CTAs/SM
//   2: 4 tiles per warp, 4 CTAs/SM
template <int K, int CB, int TG, int NT, int MINB>
static int launch_gemv_kernel(const GemvParams& prm, int sms, cudaStream_t stream)
{
    constexpr int P = 3;
    const long long units = (long long) (prm.n / 128) * (prm.k / 16);
    const int grid = (int) std::min<long long>(units, (long long) MINB * sms);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kGvThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, exl3_gemv_kernel<K, CB, TG, NT, P, MINB>, prm);
    return e == cudaSuccess ? kOk : kErrLaunch;
}

template <int K, int CB>
static int dispatch_tg(const GemvParams& prm, int sms, int variant, cudaStream_t stream)
{
    if (prm.m <= 8) {
        if (variant == 1) return launch_gemv_kernel<K, CB, 1, 4, 3>(prm, sms, stream);
        if (variant == 2) return launch_gemv_kernel<K, CB, 1, 4, 4>(prm, sms, stream);
        return launch_gemv_kernel<K, CB, 1, 8, 2>(prm, sms, stream);
    }
    if (variant == 2) return launch_gemv_kernel<K, CB, 2, 4, 3>(prm, sms, stream);
    return launch_gemv_kernel<K, CB, 2, 4, 2>(prm, sms, stream);
}

template <int K>
static int dispatch_cb(int cb, const GemvParams& prm, int sms, int variant, cudaStream_t stream)
{
    if (cb == 0) return dispatch_tg<K, 0>(prm, sms, variant, stream);
    if (cb == 1) return dispatch_tg<K, 1>(prm, sms, variant, stream);
    return dispatch_tg<K, 2>(prm, sms, variant, stream);
}

static int launch_epilogue(int cb, float* ws_acc, const __half* svh, const float* sblk, void* out,
                           long long out_stride, int out_dtype, int m, int k, int n, cudaStream_t stream)
{
    const int tasks = (n / 128) * m;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((tasks + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (cb == 2)
        e = cudaLaunchKernelEx(&cfg, exl3_gemv_epilogue_kernel<2>, ws_acc, svh, sblk, out, out_stride, out_dtype, m, k, n);
    else
        e = cudaLaunchKernelEx(&cfg, exl3_gemv_epilogue_kernel<0>, ws_acc, svh, sblk, out, out_stride, out_dtype, m, k, n);
    return e == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" size_t exl3b200_gemv_state_size(int n)
{
    if (n <= 0 || n % 128) return 0;
    return gemv_state_bytes(n);
}

extern "C" size_t exl3b200_gemv_scratch_size(int m, int k)
{
    if (m <= 0 || k <= 0 || k % 128) return 0;
    return gemv_scratch_bytes(m, k);
}

extern "C" int exl3b200_gemv(const void* x, long long x_stride, int m, int k, const void* trellis, int n, int K,
                             int cb, const void* suh, const void* svh, void* out, long long out_stride,
                             int out_dtype, int flags, void* state, size_t state_bytes, void* scratch,
                             size_t scratch_bytes, void* stream)
{
    if (!x || !trellis || !svh || !out || !state || !scratch) return kErrNullPointer;
    if (K < 2 || K > 4) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (m < 1 || m > EXL3B200_GEMV_MAX_M) return kErrBadShape;
    if (k <= 0 || n <= 0 || (k % 128) || (n % 128)) return kErrBadShape;
    if (out_dtype < 0 || out_dtype > 2) return kErrBadArgument;
    if (x_stride < k || out_stride < n) return kErrBadShape;
    const bool pre_rotated = (flags & EXL3B200_FLAG_INPUT_ROTATED) != 0;
    if (!pre_rotated && !suh) return kErrNullPointer;
    if (((uintptr_t) trellis & 3) || ((uintptr_t) x & 3) || (x_stride & 1)) return kErrUnaligned;
    if (((uintptr_t) state & 255) || ((uintptr_t) scratch & 255)) return kErrUnaligned;
    if (state_bytes < gemv_state_bytes(n) || scratch_bytes < gemv_scratch_bytes(m, k)) return kErrWorkspace;

    char* st_base = reinterpret_cast<char*>(state);
    char* sc_base = reinterpret_cast<char*>(scratch);
    float* ws_acc = reinterpret_cast<float*>(st_base);
    uint32_t* xd = reinterpret_cast<uint32_t*>(sc_base);
    float* sblk = reinterpret_cast<float*>(sc_base + align256((size_t) m * k * sizeof(uint32_t)));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    const int tasks = m * (k / 128);
    exl3_input_kernel<<<(tasks + 7) / 8, 256, 0, st>>>(
        reinterpret_cast<const __half*>(x), x_stride, reinterpret_cast<const __half*>(suh), nullptr, 0, xd,
        cb == 2 ? sblk : nullptr, m, k, pre_rotated ? 0 : 1);
    if (cudaGetLastError() != cudaSuccess) return kErrLaunch;

    GemvParams prm;
    prm.xd = xd;
    prm.trellis = reinterpret_cast<const uint32_t*>(trellis);
    prm.svh = reinterpret_cast<const __half*>(svh);
    prm.sblk = sblk;
    prm.out = out;
    prm.ws_acc = ws_acc;
    prm.out_stride = out_stride;
    prm.out_dtype = out_dtype;
    prm.m = m;
    prm.k = k;
    prm.n = n;

    const int variant = (flags >> 8) & 3;
    const int sms = sm_count();
    int rc;
    switch (K) {
        case 2: rc = dispatch_cb<2>(cb, prm, sms, variant, st); break;
        case 3: rc = dispatch_cb<3>(cb, prm, sms, variant, st); break;
        default: rc = dispatch_cb<4>(cb, prm, sms, variant, st); break;
    }
    if (rc != kOk) return rc;
    return launch_epilogue(cb, ws_acc, reinterpret_cast<const __half*>(svh), sblk, out, out_stride, out_dtype, m, k,
                           n, st);
}

extern "C" int exl3b200_hadamard_in(const void* x, long long x_stride, int m, int k, const void* suh, void* out,
                                    long long out_stride, void* stream)
{
    if (!x || !out) return kErrNullPointer;
    if (m < 1 || k <= 0 || (k % 128) || x_stride < k || out_stride < k) return kErrBadShape;
    if (((uintptr_t) x & 1) || ((uintptr_t) out & 1)) return kErrUnaligned;
    const int tasks = m * (k / 128);
    exl3_input_kernel<<<(tasks + 7) / 8, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const __half*>(x), x_stride, reinterpret_cast<const __half*>(suh),
        reinterpret_cast<__half*>(out), out_stride, nullptr, nullptr, m, k, 1);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}
