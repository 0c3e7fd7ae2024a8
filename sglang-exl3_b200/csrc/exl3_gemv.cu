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
//   tensor work is spent on padding rows.  With FOLD the codebook's final fp16
//   add (cb 0/1) is folded into the MMA: the LOP3 word {lo, hi} goes in as a k
//   pair against a duplicated activation, which saves the PRMT/HADD2 of every
//   weight pair for one extra MMA per tile.  mul1 (cb 2) feeds the exact
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
    const __half* xh;        // [M, k] fp16 rotated input (row stride k)
    const uint32_t* trellis; // [k/16, n/16, 16K] as uint32 words
    const __half* svh;       // [n]
    const float* sblk;       // [M, k/128] block sums of xh (cb 2 only)
    void* out;               // [M, out_stride]
    float* ws_acc;           // [n/128, 16, 128] zeroed fp32 partial sums
    int* ws_cnt;             // [n/128] zeroed arrival counters
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
__global__ __launch_bounds__(256) void exl3_input_kernel(
    const __half* __restrict__ x, long long x_stride, const __half* __restrict__ suh,
    __half* __restrict__ xh, long long xh_stride, float* __restrict__ sblk, int m, int k, int rotate)
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
    if (rotate) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float xv = __half2float(src[lane + 32 * i]);
            v[i] = suh ? __half2float(__float2half_rn(__fmul_rn(xv, __half2float(suh[b * 128 + lane + 32 * i]))))
                       : xv;
        }
        warp_fwht128(v, lane);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half h = __float2half_rn(__fmul_rn(v[i], kHadScale));
            xh[(size_t) row * xh_stride + b * 128 + lane + 32 * i] = h;
            v[i] = __half2float(h);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half h = src[lane + 32 * i];
            xh[(size_t) row * xh_stride + b * 128 + lane + 32 * i] = h;
            v[i] = __half2float(h);
        }
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
template <int K>
struct SliceLoad {
    static constexpr int TW = 8 * K;
    static constexpr int LOADS = (K == 3) ? 8 : (8 * TW) / 32;
};

// {lo0+hi0, lo1+hi1} from two LOP3 words, one fp16 rounding each (__hadd2)
__device__ __forceinline__ uint32_t pair_sum(uint32_t p0, uint32_t p1)
{
    const uint32_t lo = prmt(p0, p1, 0x5410);
    const uint32_t hi = prmt(p0, p1, 0x7632);
    __half2 s = __hadd2(*reinterpret_cast<const __half2*>(&lo), *reinterpret_cast<const __half2*>(&hi));
    return *reinterpret_cast<uint32_t*>(&s);
}

template <int K, int CB, int TG, bool FOLD, int P>
__global__ __launch_bounds__(kGvThreads, 2) void exl3_gemv_kernel(const GemvParams p)
{
    constexpr int TW = SliceLoad<K>::TW;
    constexpr int LOADS = SliceLoad<K>::LOADS;
    constexpr bool USE_FOLD = FOLD || CB == 2;

    __shared__ float red[TG * 8][kRedStride];
    __shared__ int s_last;

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

    // lane load predicate (K = 3: 24 of 32 lanes carry a tile's words)
    const bool load_lane = (K != 3) || lane < 24;

    bool waited = false;

    for (long long u = u_begin; u < u_end;) {
        const int nb = (int) (u / kt_total);
        const int kr0 = (int) (u - (long long) nb * kt_total);
        const int len = (int) min((long long) (kt_total - kr0), u_end - u);

        for (int i = threadIdx.x; i < TG * 8 * kRedStride; i += kGvThreads) (&red[0][0])[i] = 0.f;

        float acc[8][TG][4];
#pragma unroll
        for (int t = 0; t < 8; ++t)
#pragma unroll
            for (int q = 0; q < TG; ++q)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[t][q][r] = 0.f;

        // slices of this warp: kr0 + warp + kGvWarps * i, i < nr
        const int nr = len > warp ? (len - warp + kGvWarps - 1) / kGvWarps : 0;

        auto slice_ptr = [&](int i) -> const uint32_t* {
            const int kr = kr0 + warp + kGvWarps * i;
            return p.trellis + ((size_t) kr * n_tiles + (size_t) nb * 8) * TW;
        };
        auto load_slice = [&](int i, uint32_t (&dst)[LOADS]) {
            const uint32_t* bp = slice_ptr(i);
#pragma unroll
            for (int l = 0; l < LOADS; ++l) {
                const int off = (K == 3) ? l * TW + lane : l * 32 + lane;
                dst[l] = load_lane ? __ldcs(bp + off) : 0u;
            }
        };
        auto load_x = [&](int i, uint32_t (&xb)[TG][2]) {
            const int kr = kr0 + warp + kGvWarps * i;
#pragma unroll
            for (int q = 0; q < TG; ++q) {
                const int row = 8 * q + g;
                if (row < p.m) {
                    const uint32_t* xr = reinterpret_cast<const uint32_t*>(p.xh + (size_t) row * p.k + kr * 16);
                    xb[q][0] = __ldcg(xr + c);
                    xb[q][1] = __ldcg(xr + c + 4);
                } else {
                    xb[q][0] = 0u;
                    xb[q][1] = 0u;
                }
            }
        };

        uint32_t ring[P][LOADS];
#pragma unroll
        for (int s = 0; s < P; ++s)
            if (s < nr) load_slice(s, ring[s]);

        if (!waited) {
            griddep_wait();
            waited = true;
        }

        uint32_t xring[P][TG][2];
#pragma unroll
        for (int s = 0; s < P; ++s)
            if (s < nr) load_x(s, xring[s]);

        for (int i0 = 0; i0 < nr; i0 += P) {
#pragma unroll
            for (int s = 0; s < P; ++s) {
                const int i = i0 + s;
                if (i >= nr) break;
                uint32_t bw[LOADS];
                uint32_t xb[TG][2];
#pragma unroll
                for (int l = 0; l < LOADS; ++l) bw[l] = ring[s][l];
#pragma unroll
                for (int q = 0; q < TG; ++q) {
                    xb[q][0] = xring[s][q][0];
                    xb[q][1] = xring[s][q][1];
                }
                if (i + P < nr) {
                    load_slice(i + P, ring[s]);
                    load_x(i + P, xring[s]);
                }

                // folded activation fragments: {x, x} pairs
                uint32_t xf[TG][4];
                if constexpr (USE_FOLD) {
#pragma unroll
                    for (int q = 0; q < TG; ++q) {
                        xf[q][0] = prmt(xb[q][0], 0u, 0x1010);  // x[2c]   duplicated
                        xf[q][1] = prmt(xb[q][0], 0u, 0x3232);  // x[2c+1] duplicated
                        xf[q][2] = prmt(xb[q][1], 0u, 0x1010);  // x[2c+8]
                        xf[q][3] = prmt(xb[q][1], 0u, 0x3232);  // x[2c+9]
                    }
                }

#pragma unroll
                for (int t = 0; t < 8; ++t) {
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

                    if constexpr (USE_FOLD) {
                        const uint32_t aA[4] = {pv[0], pv[4], pv[1], pv[5]};
                        const uint32_t aB[4] = {pv[2], pv[6], pv[3], pv[7]};
#pragma unroll
                        for (int q = 0; q < TG; ++q) {
                            mma_16816(aA, xf[q][0], xf[q][1], acc[t][q]);
                            mma_16816(aB, xf[q][2], xf[q][3], acc[t][q]);
                        }
                    } else {
                        // pairs (j0,j1) (j4,j5) (j2,j3) (j6,j7): lo+hi with one fp16 rounding
                        const uint32_t v[4] = {pair_sum(pv[0], pv[1]), pair_sum(pv[4], pv[5]),
                                               pair_sum(pv[2], pv[3]), pair_sum(pv[6], pv[7])};
#pragma unroll
                        for (int q = 0; q < TG; ++q) mma_16816(v, xb[q][0], xb[q][1], acc[t][q]);
                    }
                }
            }
        }

        if (!waited) {
            griddep_wait();
            waited = true;
        }
        __syncthreads();  // red zeroed by all threads before any atomics

        // fragment -> shared block: lane holds (n = 16t + g (+8), rows 8q + 2c (+1))
#pragma unroll
        for (int q = 0; q < TG; ++q) {
            const int r0 = 8 * q + 2 * c;
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                if (r0 < p.m) {
                    atomicAdd(&red[r0][16 * t + g], acc[t][q][0]);
                    atomicAdd(&red[r0][16 * t + g + 8], acc[t][q][2]);
                }
                if (r0 + 1 < p.m) {
                    atomicAdd(&red[r0 + 1][16 * t + g], acc[t][q][1]);
                    atomicAdd(&red[r0 + 1][16 * t + g + 8], acc[t][q][3]);
                }
            }
        }
        __syncthreads();

        bool do_epilogue = (kr0 == 0 && len == kt_total);
        if (!do_epilogue) {
            float* wsb = p.ws_acc + (size_t) nb * 16 * 128;
            for (int i = threadIdx.x; i < p.m * 128; i += kGvThreads) {
                const int r = i >> 7, col = i & 127;
                atomicAdd(wsb + r * 128 + col, red[r][col]);
            }
            __threadfence();
            __syncthreads();
            if (threadIdx.x == 0) {
                const long long uf = (long long) nb * kt_total;
                const long long ul = uf + kt_total - 1;
                const long long of = ((uf + 1) * G - 1) / units;
                const long long ol = ((ul + 1) * G - 1) / units;
                const int contributors = (int) (ol - of + 1);
                const int prev = atomicAdd(p.ws_cnt + nb, 1);
                s_last = (prev == contributors - 1);
            }
            __syncthreads();
            do_epilogue = s_last != 0;
            if (do_epilogue) {
                __threadfence();
                for (int i = threadIdx.x; i < p.m * 128; i += kGvThreads) {
                    const int r = i >> 7, col = i & 127;
                    red[r][col] = __ldcg(wsb + r * 128 + col);
                    wsb[r * 128 + col] = 0.f;
                }
                if (threadIdx.x == 0) p.ws_cnt[nb] = 0;
                __syncthreads();
            }
        }

        if (do_epilogue) {
            float k_inv = 0.f, k_bias = 0.f;
            if constexpr (CB == 2) {
                k_inv = __half2float(__ushort_as_half(kMul1InvBits));
                k_bias = __half2float(__ushort_as_half(kMul1BiasBits));
            }
            for (int r = warp; r < p.m; r += kGvWarps) {
                float v[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = red[r][lane + 32 * i];
                if constexpr (CB == 2) {
                    const int nblk = p.k >> 7;
                    float s = 0.f;
                    for (int b = lane; b < nblk; b += 32) s += __ldcg(p.sblk + (size_t) r * nblk + b);
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
#pragma unroll
                    for (int i = 0; i < 4; ++i) v[i] = fmaf(k_inv, v[i], k_bias * s);
                }
                warp_fwht128(v, lane);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int col = nb * 128 + lane + 32 * i;
                    const float y = v[i] * kHadScale * __half2float(p.svh[col]);
                    store_out(p.out, (size_t) r * p.out_stride + col, y, p.out_dtype);
                }
            }
        }
        __syncthreads();
        u += len;
    }
    if (!waited) griddep_wait();
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

// state: [n/128][16][128] fp32 partial sums, then [n/128] int arrival counters;
// zero when allocated, left zero by every call.
static size_t gemv_state_bytes(int n)
{
    const size_t nblocks = (size_t) n / 128;
    return align256(nblocks * 16 * 128 * sizeof(float)) + align256(nblocks * sizeof(int));
}

// scratch: [m][k] fp16 rotated input, then [m][k/128] fp32 block sums.
static size_t gemv_scratch_bytes(int m, int k)
{
    return align256((size_t) m * k * sizeof(__half)) + align256((size_t) m * (k / 128) * sizeof(float));
}

template <int K, int CB, int TG, bool FOLD>
static int launch_gemv_kernel(const GemvParams& prm, int grid, cudaStream_t stream)
{
    constexpr int P = TG == 1 ? 3 : 2;
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
    cudaError_t e = cudaLaunchKernelEx(&cfg, exl3_gemv_kernel<K, CB, TG, FOLD, P>, prm);
    return e == cudaSuccess ? kOk : kErrLaunch;
}

template <int K, int CB>
static int dispatch_tg(const GemvParams& prm, int grid, bool fold, cudaStream_t stream)
{
    if (prm.m <= 8) {
        if (fold) return launch_gemv_kernel<K, CB, 1, true>(prm, grid, stream);
        return launch_gemv_kernel<K, CB, 1, false>(prm, grid, stream);
    }
    if (fold) return launch_gemv_kernel<K, CB, 2, true>(prm, grid, stream);
    return launch_gemv_kernel<K, CB, 2, false>(prm, grid, stream);
}

template <int K>
static int dispatch_cb(int cb, const GemvParams& prm, int grid, bool fold, cudaStream_t stream)
{
    if (cb == 0) return dispatch_tg<K, 0>(prm, grid, fold, stream);
    if (cb == 1) return dispatch_tg<K, 1>(prm, grid, fold, stream);
    return dispatch_tg<K, 2>(prm, grid, true, stream);
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
    int* ws_cnt = reinterpret_cast<int*>(st_base + align256((size_t) (n / 128) * 16 * 128 * sizeof(float)));
    __half* xh = reinterpret_cast<__half*>(sc_base);
    float* sblk = reinterpret_cast<float*>(sc_base + align256((size_t) m * k * sizeof(__half)));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);

    const int tasks = m * (k / 128);
    exl3_input_kernel<<<(tasks + 7) / 8, 256, 0, st>>>(
        reinterpret_cast<const __half*>(x), x_stride, reinterpret_cast<const __half*>(suh), xh, k,
        cb == 2 ? sblk : nullptr, m, k, pre_rotated ? 0 : 1);
    if (cudaGetLastError() != cudaSuccess) return kErrLaunch;

    GemvParams prm;
    prm.xh = xh;
    prm.trellis = reinterpret_cast<const uint32_t*>(trellis);
    prm.svh = reinterpret_cast<const __half*>(svh);
    prm.sblk = sblk;
    prm.out = out;
    prm.ws_acc = ws_acc;
    prm.ws_cnt = ws_cnt;
    prm.out_stride = out_stride;
    prm.out_dtype = out_dtype;
    prm.m = m;
    prm.k = k;
    prm.n = n;

    const long long units = (long long) (n / 128) * (k / 16);
    const int grid = (int) std::min<long long>(units, (long long) 2 * sm_count());
    const bool fold = (flags & EXL3B200_FLAG_NO_FOLD) == 0;
    switch (K) {
        case 2: return dispatch_cb<2>(cb, prm, grid, fold, st);
        case 3: return dispatch_cb<3>(cb, prm, grid, fold, st);
        default: return dispatch_cb<4>(cb, prm, grid, fold, st);
    }
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
        reinterpret_cast<__half*>(out), out_stride, nullptr, m, k, 1);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}
