// Small-M EXL3 matmul (m <= 16 rows per problem), grouped over a table of
// problems: y = H128(H128(x * suh) @ W_raw) * svh / 128 for every problem.
//
// Replaces the reference's cooperative QTIP-style GEMV
// (csrc/quant/exl3_gemv_kernel.cuh:138-402, host csrc/exl3_gemv.cu:26-63), its
// per-expert batched form (csrc/p2b_batched.cu:13-101) and the row chunks of
// exl3_gemm (csrc/exl3_gemm.cu:9-31) with three kernels chained by programmatic
// dependent launch (PDL), none of which waits on another CTA:
//
// * input stage (exl3_gv_input_kernel): one warp per (problem, row, 128-block)
//   computes the fp16 x_had = H128(x * suh) / sqrt(128) with the reference's
//   roundings (had_hf_r_128_inner<true,false>, csrc/quant/hadamard_inner.cuh:93-147)
//   and stores it as duplicated pairs {h, h}: the B fragments of the folded MMA.
// * matmul (exl3_gv_matmul_kernel): the iteration space is every problem's list
//   of units (128-column block nb, 16-row k-slice kr); the grid (2 CTAs per SM)
//   splits the concatenated list evenly ("stream-K"), so any mix of shapes
//   load-balances over the 148 SMs.  Each warp of a CTA takes k-slices of the
//   current block and, per slice, streams the block's tiles with coalesced 32-bit
//   loads (one 128-byte transaction per tile at 4 bpw) through a register ring
//   three slices deep, resolves each lane's two stream words with shuffles,
//   extracts the 8 windows and runs the codebook in registers.  The decoded 16x16
//   tile is used transposed as the A operand of mma.m16n8k16 (rows = output
//   columns, cols = k) and x_had as B (k x 8 rows), fp32 accumulate, so at m <= 8
//   no tensor work is spent on padding rows.  The codebook's final fp16 add
//   (cb 0/1) is folded into the MMA: the LOP3 word {lo, hi} goes in as a k pair
//   against the duplicated activation.  mul1 (cb 2) feeds the exact
//   integer-valued fp16 h = 1024 + bytesum; the epilogue applies
//   y = k_inv * sum(x h) + k_bias * sum(x).  The integer-logic and IMAD pipes
//   (both half rate on sm_100) bound the decode, so window extraction uses byte
//   permutes and shifts the compiler can place on either pipe.  Warps reduce
//   their fragments in shared memory and the CTA adds its partial block into a
//   zeroed fp32 state slice with fire-and-forget atomics, then moves on.
// * epilogue (exl3_gv_epilogue_kernel): one warp per (problem, 128-column block,
//   row) reads the summed partials and re-zeroes them, runs H128 over the block,
//   * 1/sqrt(128) * svh, and then stores (fp16 / bf16 / fp32), or adds
//   weight * y into a routed fp32 output row (MoE combine), or - for (gate, up)
//   problem pairs - applies the clipped SwiGLU and writes the rotated input of the
//   down projection (the reference's had_hf_r_128_guad_inner and p2b_moe phase 3,
//   csrc/quant/hadamard_inner.cuh:283-413, csrc/p2b_moe.cu:300-336).
#include <algorithm>
#include <atomic>

#include "exl3_common.cuh"
#include "exl3_capi_internal.h"
#include "exl3_grouped.cuh"
#include "exl3_grouped_dev.cuh"
#include "exl3_epilogue.cuh"

namespace exl3b200 {

constexpr int kGvThreads = 256;
constexpr int kGvWarps = kGvThreads / 32;
constexpr int kRedStride = 132;  // padded row stride of the shared reduction block

// ---------------------------------------------------------------------------
// input stage
// ---------------------------------------------------------------------------

__global__ __launch_bounds__(256) void exl3_gv_input_kernel(const __grid_constant__ GvArgs a)
{
    griddep_launch();
    griddep_wait();  // inputs may be produced by the previous kernel (no-op otherwise)
    const GvTotals tot = gv_totals(a);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < tot.in_tasks; task += warps) {
        const int pi = gv_find<0>(a, tot.nprob, task);
        const GvProblem& p = gv_prob(a, pi);
        const int nblk = p.k >> 7;
        const int local = task - p.in_task_begin;
        const int r = local / nblk;
        const int b = local - r * nblk;
        const int row = p.x_rows ? p.x_rows[r] : r;
        __half h[4];
        rotate_block(p.x + (size_t) row * p.x_stride + b * 128, p.suh ? p.suh + b * 128 : nullptr, lane, h);
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t u = __half_as_ushort(h[i]);
            p.xd[(size_t) r * p.k + b * 128 + lane + 32 * i] = u | (u << 16);
            s += __half2float(h[i]);
        }
        if (p.sblk) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0) p.sblk[(size_t) r * nblk + b] = s;
        }
    }
}

// ---------------------------------------------------------------------------
// matmul
// ---------------------------------------------------------------------------

// Loads per k-slice per lane for a warp's NT tiles: tiles are 8K words; K = 1, 2, 4
// pack 32/(8K) tiles into one 32-lane load, K = 3 loads one tile per load on 24 lanes.
template <int K, int NT>
struct SliceLoad {
    static constexpr int TW = 8 * K;
    static constexpr int LOADS = (K == 3) ? NT : (NT * TW) / 32;
};

// K bits, codebook CB, TG groups of 8 rows, NT tiles per warp per k-slice (8 or 4:
// with 4, two warps share a slice's 8-tile block), P-deep trellis register ring.
template <int K, int CB, int TG, int NT, int P, int MINB>
__global__ __launch_bounds__(kGvThreads, MINB) void exl3_gv_matmul_kernel(const __grid_constant__ GvArgs a)
{
    griddep_launch();  // let the epilogue kernel get scheduled early; it waits for this grid
    constexpr int TW = SliceLoad<K, NT>::TW;
    constexpr int LOADS = SliceLoad<K, NT>::LOADS;
    constexpr int TGRP = 8 / NT;         // warps sharing one slice
    constexpr int SG = kGvWarps / TGRP;  // slice groups

    __shared__ float red[SG][TG * 8][kRedStride];  // per slice group: its warps' partial block

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int c = lane & 3;
    const LaneWords lw = lane_words<K>(lane);
    const bool load_lane = (K != 3) || lane < 24;  // K = 3: 24 of 32 lanes carry a tile's words

    bool waited = false;
    if (a.dev_totals) {  // the totals are produced by an earlier kernel
        griddep_wait();
        waited = true;
    }
    const GvTotals tot = gv_totals(a);
    const long long units = tot.units;
    const long long G = gridDim.x;
    long long u_begin, u_end;
    if (a.cta_per_block > 0) {
        // block-aligned split: cta_per_block CTAs share each 128-column block's k
        // range (every problem has a.block_units k-slices), no CTA crosses a block
        const long long blk = blockIdx.x / a.cta_per_block;
        const int j = blockIdx.x - (int) blk * a.cta_per_block;
        u_begin = blk * a.block_units + (long long) j * a.block_units / a.cta_per_block;
        u_end = blk * a.block_units + (long long) (j + 1) * a.block_units / a.cta_per_block;
    } else {
        u_begin = (long long) blockIdx.x * units / G;
        u_end = (long long) (blockIdx.x + 1) * units / G;
    }

    int pi = -1;
    long long pu0 = 0, pu1 = 0;  // unit range of the current problem
    for (long long u = u_begin; u < u_end;) {
        if (u >= pu1) {
            pi = a.uniform_units > 0 ? (int) (u / a.uniform_units) : gv_find<2>(a, tot.nprob, (int) u);
            const GvProblem& pp = gv_prob(a, pi);
            pu0 = a.uniform_units > 0 ? (long long) pi * a.uniform_units : pp.unit_begin;
            pu1 = pu0 + (long long) (pp.n >> 7) * (pp.k >> 4);
        }
        const GvProblem& p = gv_prob(a, pi);
        const int kt_total = p.k >> 4;
        const int n_tiles = p.n >> 4;
        const long long lu = u - pu0;
        const int nb = (int) (lu / kt_total);
        const int kr0 = (int) (lu - (long long) nb * kt_total);
        const int len = (int) min((long long) (kt_total - kr0), u_end - u);
        const int m = p.m;
        const size_t slice_words = (size_t) n_tiles * TW;  // words per k-slice row of the matrix

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
            xrow[q] = row < m;
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
                    // a row group past the problem's rows would only add zeros (its
                    // activations are zero): skip its MMAs (warp-uniform per problem)
                    if (q > 0 && 8 * q >= m) break;
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

        // fragments -> the slice group's partial block (lane holds n = 16t + g (+8),
        // rows 8q + 2c (+1)); the previous segment's readers passed the barrier below
#pragma unroll
        for (int q = 0; q < TG; ++q) {
            const int r0 = 8 * q + 2 * c;
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const int n0 = 16 * (th * NT + t) + g;
                if (r0 < m) {
                    red[sg][r0][n0] = acc[t][q][0];
                    red[sg][r0][n0 + 8] = acc[t][q][2];
                }
                if (r0 + 1 < m) {
                    red[sg][r0 + 1][n0] = acc[t][q][1];
                    red[sg][r0 + 1][n0 + 8] = acc[t][q][3];
                }
            }
        }
        __syncthreads();

        // sum over the slice groups, then fire-and-forget: add this CTA's partial block
        // into the zeroed state; the epilogue kernel (a programmatic dependent of this
        // grid) finishes it
        float* wsb = p.acc + (size_t) nb * p.acc_nb_stride;
        for (int e = threadIdx.x; e < m * 128; e += kGvThreads) {
            const int r = e >> 7, col = e & 127;
            float s = red[0][r][col];
#pragma unroll
            for (int j = 1; j < SG; ++j) s += red[j][r][col];
            atomicAdd(wsb + r * 128 + col, s);
        }
        __syncthreads();
        u += len;
    }
    if (!waited) griddep_wait();
}

// ---------------------------------------------------------------------------
// epilogue
// ---------------------------------------------------------------------------

// Finish one (problem, block, row): read and re-zero the summed partials, mul1
// correction, H128, * 1/sqrt(128) * svh.  Lane holds columns lane + 32 i.
template <int CB, int MODE>
__global__ __launch_bounds__(256) void exl3_gv_epilogue_kernel(const __grid_constant__ GvArgs a)
{
    griddep_launch();
    const int lane = threadIdx.x & 31;
    gv_prefetch_epilogue(a, lane);
    griddep_wait();
    const GvTotals tot = gv_totals(a);
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < tot.out_tasks; task += warps) {
        const int pi = gv_find<1>(a, tot.nprob, task);
        const GvProblem& p = gv_prob(a, pi);
        const int nblocks = p.n >> 7;
        const int local = task - p.out_task_begin;
        const int r = local / nblocks;
        const int nb = local - r * nblocks;
        if constexpr (MODE == kEpiSwiglu) {
            // (gate, up) pair: table entries j and j+1 (stride 2 view)
            const GvProblem& pu = a.dev ? a.dev[pi * a.stride + a.offset + 1] : a.inl[pi * a.stride + a.offset + 1];
            epi_block_row<CB>(a, DecAux{}, MODE, pi, p, &pu, nb, r, lane);
        } else if constexpr (MODE == kEpiSwigluFused) {
            // one gate|up problem: gate block nb with up block nb + n / 256; the task
            // grid counts n / 256 blocks per row
            const int half = p.n >> 8;
            const int r2 = local / half, nb2 = local - r2 * half;
            GvProblem pd = p;
            pd.n = p.n >> 1;  // the down projection's input width, for the output's indexing
            const EpiPre ep = epi_preload(p, DecAux{}, kEpiSwiglu, pi, nb2, r2, lane);
            float v[4], u[4];
            gv_finish<CB>(p, nb2, r2, lane, v);
            gv_finish<CB>(p, nb2 + half, r2, lane, u);
            epi_apply<CB>(a, DecAux{}, kEpiSwiglu, pi, pd, nb2, r2, lane, v, u, ep);
        } else {
            epi_block_row<CB>(a, DecAux{}, MODE, pi, p, nullptr, nb, r, lane);
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

int gv_sm_count()
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

size_t gv_state_bytes_per_problem(int n) { return align256((size_t) (n / 128) * 16 * 128 * sizeof(float)); }
size_t gv_xd_bytes(int m, int k) { return align256((size_t) m * k * sizeof(uint32_t)); }
size_t gv_sblk_bytes(int m, int k) { return align256((size_t) m * (k / 128) * sizeof(float)); }

template <typename Kern>
static int launch_ex(Kern kern, int grid, bool pdl, cudaStream_t stream, const GvArgs& a)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::max(grid, 1));
    cfg.blockDim = dim3(kGvThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? kOk : kErrLaunch;
}

int gv_launch_input(const GvArgs& a, int max_in_tasks, bool pdl, cudaStream_t stream)
{
    const int warps_per_cta = kGvThreads / 32;
    const int grid = std::min((max_in_tasks + warps_per_cta - 1) / warps_per_cta, 8 * gv_sm_count());
    return launch_ex(exl3_gv_input_kernel, grid, pdl, stream, a);
}

// Tiling variants (the kernel-shape map picks one per call):
//   0: 8 tiles per warp, 2 CTAs/SM    1: 4 tiles per warp, 3 CTAs/SM
// A CTA whose unit range crosses into another 128-column block pays a second
// reduction and a cold start of its trellis loads (~3 us, about 20 units of
// streaming at this grid).  For a host-built table whose problems share k, when
// few blocks share the grid, splitting each block's k range over a whole number
// of CTAs removes the crossings; the host takes it when its per-CTA units do not
// exceed stream-K's plus that penalty.
constexpr int kCrossPenaltyUnits = 20;

static int block_aligned_split(GvArgs& a, int grid)
{
    if (a.dev || a.dev_totals || a.uniform_units > 0 || a.stride != 1 || a.offset != 0 || a.nprob < 1) return grid;
    const int k = a.inl[0].k;
    long long blocks = 0;
    for (int i = 0; i < a.nprob; ++i) {
        if (a.inl[i].k != k) return grid;
        blocks += a.inl[i].n / 128;
    }
    const int kt = k / 16;
    if (blocks < 1 || blocks > grid) return grid;
    const int cpb = std::min<long long>(grid / blocks, kt);
    const long long aligned = (kt + cpb - 1) / cpb;
    const long long stream_k = (a.units + grid - 1) / grid + kCrossPenaltyUnits;
    if (aligned > stream_k) return grid;
    a.cta_per_block = cpb;
    a.block_units = kt;
    return (int) (blocks * cpb);
}

template <int K, int CB, int TG, int NT, int MINB>
static int launch_matmul_t(const GvArgs& a_in, bool pdl, cudaStream_t stream)
{
    constexpr int P = 3;
    GvArgs a = a_in;
    a.cta_per_block = 0;
    int grid = MINB * gv_sm_count();
    if (!a.dev_totals) {
        const long long units = a.uniform_units > 0 ? (long long) a.nprob * a.uniform_units : a.units;
        grid = (int) std::min<long long>(units, grid);
        grid = block_aligned_split(a, grid);
    }
    return launch_ex(exl3_gv_matmul_kernel<K, CB, TG, NT, P, MINB>, grid, pdl, stream, a);
}

template <int K, int CB>
static int launch_matmul_tg(const GvArgs& a, int max_rows, int variant, bool pdl, cudaStream_t stream)
{
    if (max_rows <= 8) {
        if (variant == 1) return launch_matmul_t<K, CB, 1, 4, 3>(a, pdl, stream);
        return launch_matmul_t<K, CB, 1, 8, 2>(a, pdl, stream);
    }
    return launch_matmul_t<K, CB, 2, 4, 2>(a, pdl, stream);
}

template <int K>
static int launch_matmul_cb(const GvArgs& a, int cb, int max_rows, int variant, bool pdl, cudaStream_t stream)
{
    if (cb == 0) return launch_matmul_tg<K, 0>(a, max_rows, variant, pdl, stream);
    if (cb == 1) return launch_matmul_tg<K, 1>(a, max_rows, variant, pdl, stream);
    return launch_matmul_tg<K, 2>(a, max_rows, variant, pdl, stream);
}

int gv_launch_matmul(const GvArgs& a, int K, int cb, int max_rows, int variant, bool pdl, cudaStream_t stream)
{
    switch (K) {
        case 2: return launch_matmul_cb<2>(a, cb, max_rows, variant, pdl, stream);
        case 3: return launch_matmul_cb<3>(a, cb, max_rows, variant, pdl, stream);
        case 4: return launch_matmul_cb<4>(a, cb, max_rows, variant, pdl, stream);
        default: return kErrBadBits;
    }
}

int gv_launch_epilogue(const GvArgs& a, int cb, int max_out_tasks, bool pdl, cudaStream_t stream)
{
    const int warps_per_cta = kGvThreads / 32;
    const int grid = std::min((max_out_tasks + warps_per_cta - 1) / warps_per_cta, 8 * gv_sm_count());
    const bool mul1 = cb == 2;
    switch (a.epi_mode) {
        case kEpiStore:
            return mul1 ? launch_ex(exl3_gv_epilogue_kernel<2, kEpiStore>, grid, pdl, stream, a)
                        : launch_ex(exl3_gv_epilogue_kernel<0, kEpiStore>, grid, pdl, stream, a);
        case kEpiCombine:
            return mul1 ? launch_ex(exl3_gv_epilogue_kernel<2, kEpiCombine>, grid, pdl, stream, a)
                        : launch_ex(exl3_gv_epilogue_kernel<0, kEpiCombine>, grid, pdl, stream, a);
        case kEpiSwiglu:
            return mul1 ? launch_ex(exl3_gv_epilogue_kernel<2, kEpiSwiglu>, grid, pdl, stream, a)
                        : launch_ex(exl3_gv_epilogue_kernel<0, kEpiSwiglu>, grid, pdl, stream, a);
        case kEpiSwigluFused:
            return mul1 ? launch_ex(exl3_gv_epilogue_kernel<2, kEpiSwigluFused>, grid, pdl, stream, a)
                        : launch_ex(exl3_gv_epilogue_kernel<0, kEpiSwigluFused>, grid, pdl, stream, a);
        default: return kErrBadArgument;
    }
}

void gv_prefix_inline(GvArgs& a)
{
    int units = 0, in_tasks = 0, out_tasks = 0;
    for (int i = 0; i < a.nprob; ++i) {
        GvProblem& p = a.inl[i];
        p.unit_begin = units;
        p.in_task_begin = in_tasks;
        p.out_task_begin = out_tasks;
        units += (p.n / 128) * (p.k / 16);
        in_tasks += p.m * (p.k / 128);
        out_tasks += p.m * (p.n / 128);
    }
    a.units = units;
    a.in_tasks = in_tasks;
    a.out_tasks = out_tasks;
    a.dev = nullptr;
    a.dev_totals = nullptr;
    a.stride = 1;
    a.offset = 0;
    a.uniform_units = 0;
}

// Host-built table of up to kGvInline dense problems (one input matrix, several
// linears sharing K and codebook): fill prefixes and launch the three kernels.
static int run_inline(GvArgs& a, int K, int cb, int max_rows, int variant, cudaStream_t stream)
{
    gv_prefix_inline(a);
    int rc = gv_launch_input(a, a.in_tasks, false, stream);
    if (rc != kOk) return rc;
    rc = gv_launch_matmul(a, K, cb, max_rows, variant, true, stream);
    if (rc != kOk) return rc;
    return gv_launch_epilogue(a, cb, a.out_tasks, true, stream);
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" size_t exl3b200_gemv_state_size(int n)
{
    if (n <= 0 || n % 128) return 0;
    return gv_state_bytes_per_problem(n);
}

extern "C" size_t exl3b200_gemv_scratch_size(int m, int k)
{
    if (m <= 0 || k <= 0 || k % 128) return 0;
    return gv_xd_bytes(m, k) + gv_sblk_bytes(m, k);
}

static int check_linear_args(const void* trellis, const void* svh, int m, int k, int n, int K, int cb)
{
    if (!trellis || !svh) return kErrNullPointer;
    if (K < 2 || K > 4) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (m < 1 || m > EXL3B200_GEMV_MAX_M) return kErrBadShape;
    if (k <= 0 || n <= 0 || (k % 128) || (n % 128)) return kErrBadShape;
    if ((uintptr_t) trellis & 3) return kErrUnaligned;
    return kOk;
}

extern "C" int exl3b200_gemv(const void* x, long long x_stride, int m, int k, const void* trellis, int n, int K,
                             int cb, const void* suh, const void* svh, void* out, long long out_stride,
                             int out_dtype, int flags, void* state, size_t state_bytes, void* scratch,
                             size_t scratch_bytes, void* stream)
{
    if (!x || !out || !state || !scratch) return kErrNullPointer;
    int rc = check_linear_args(trellis, svh, m, k, n, K, cb);
    if (rc != kOk) return rc;
    if (out_dtype < 0 || out_dtype > 2) return kErrBadArgument;
    if (x_stride < k || out_stride < n) return kErrBadShape;
    const bool pre_rotated = (flags & EXL3B200_FLAG_INPUT_ROTATED) != 0;
    if (!pre_rotated && !suh) return kErrNullPointer;
    if (((uintptr_t) x & 3) || (x_stride & 1)) return kErrUnaligned;
    if (((uintptr_t) state & 255) || ((uintptr_t) scratch & 255)) return kErrUnaligned;
    if (state_bytes < gv_state_bytes_per_problem(n) || scratch_bytes < gv_xd_bytes(m, k) + gv_sblk_bytes(m, k))
        return kErrWorkspace;

    GvArgs a = {};
    a.nprob = 1;
    a.out_dtype = out_dtype;
    a.epi_mode = kEpiStore;
    GvProblem& p = a.inl[0];
    p.trellis = reinterpret_cast<const uint32_t*>(trellis);
    p.suh = pre_rotated ? nullptr : reinterpret_cast<const __half*>(suh);
    p.svh = reinterpret_cast<const __half*>(svh);
    p.x = reinterpret_cast<const __half*>(x);
    p.x_stride = x_stride;
    p.xd = reinterpret_cast<uint32_t*>(scratch);
    p.sblk = cb == 2 ? reinterpret_cast<float*>(reinterpret_cast<char*>(scratch) + gv_xd_bytes(m, k)) : nullptr;
    p.acc = reinterpret_cast<float*>(state);
    p.acc_nb_stride = 16 * 128;
    p.out = out;
    p.out_stride = out_stride;
    p.k = k;
    p.n = n;
    p.m = m;
    return run_inline(a, K, cb, m, (flags >> 8) & 3, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int exl3b200_gemv_multi(int count, const void* x, long long x_stride, int m, int k, int K, int cb,
                                   const void* const* trellis, const int* n, const void* const* suh,
                                   const void* const* svh, void* const* out, const long long* out_stride,
                                   int out_dtype, int flags, void* state, size_t state_bytes, void* scratch,
                                   size_t scratch_bytes, void* stream)
{
    if (count < 1 || count > EXL3B200_MULTI_MAX) return kErrBadArgument;
    if (!x || !trellis || !n || !suh || !svh || !out || !out_stride || !state || !scratch) return kErrNullPointer;
    if (out_dtype < 0 || out_dtype > 2) return kErrBadArgument;
    if (x_stride < k || ((uintptr_t) x & 3) || (x_stride & 1)) return kErrUnaligned;
    if (((uintptr_t) state & 255) || ((uintptr_t) scratch & 255)) return kErrUnaligned;
    size_t need_state = 0, need_scratch = 0;
    for (int i = 0; i < count; ++i) {
        int rc = check_linear_args(trellis[i], svh[i], m, k, n[i], K, cb);
        if (rc != kOk) return rc;
        if (!suh[i] || !out[i]) return kErrNullPointer;
        if (out_stride[i] < n[i]) return kErrBadShape;
        need_state += gv_state_bytes_per_problem(n[i]);
        need_scratch += gv_xd_bytes(m, k) + gv_sblk_bytes(m, k);
    }
    if (state_bytes < need_state || scratch_bytes < need_scratch) return kErrWorkspace;

    GvArgs a = {};
    a.nprob = count;
    a.out_dtype = out_dtype;
    a.epi_mode = kEpiStore;
    char* st = reinterpret_cast<char*>(state);
    char* sc = reinterpret_cast<char*>(scratch);
    for (int i = 0; i < count; ++i) {
        GvProblem& p = a.inl[i];
        p.trellis = reinterpret_cast<const uint32_t*>(trellis[i]);
        p.suh = reinterpret_cast<const __half*>(suh[i]);
        p.svh = reinterpret_cast<const __half*>(svh[i]);
        p.x = reinterpret_cast<const __half*>(x);
        p.x_stride = x_stride;
        p.xd = reinterpret_cast<uint32_t*>(sc);
        sc += gv_xd_bytes(m, k);
        p.sblk = cb == 2 ? reinterpret_cast<float*>(sc) : nullptr;
        sc += gv_sblk_bytes(m, k);
        p.acc = reinterpret_cast<float*>(st);
        p.acc_nb_stride = 16 * 128;
        st += gv_state_bytes_per_problem(n[i]);
        p.out = out[i];
        p.out_stride = out_stride[i];
        p.k = k;
        p.n = n[i];
        p.m = m;
    }
    return run_inline(a, K, cb, m, (flags >> 8) & 3, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int exl3b200_gemv_combine(const void* x, long long x_stride, int m, int k, const void* trellis, int n,
                                     int K, int cb, const void* suh, const void* svh, float* out,
                                     long long out_stride, const int* out_rows, const float* out_scale, int flags,
                                     void* state, size_t state_bytes, void* scratch, size_t scratch_bytes,
                                     void* stream)
{
    if (!x || !out || !out_rows || !state || !scratch) return kErrNullPointer;
    int rc = check_linear_args(trellis, svh, m, k, n, K, cb);
    if (rc != kOk) return rc;
    if (x_stride < k || out_stride < n) return kErrBadShape;
    const bool pre_rotated = (flags & EXL3B200_FLAG_INPUT_ROTATED) != 0;
    if (!pre_rotated && !suh) return kErrNullPointer;
    if (((uintptr_t) x & 3) || (x_stride & 1)) return kErrUnaligned;
    if (((uintptr_t) state & 255) || ((uintptr_t) scratch & 255)) return kErrUnaligned;
    if (state_bytes < gv_state_bytes_per_problem(n) || scratch_bytes < gv_xd_bytes(m, k) + gv_sblk_bytes(m, k))
        return kErrWorkspace;
    GvArgs a = {};
    a.nprob = 1;
    a.epi_mode = kEpiCombine;
    GvProblem& p = a.inl[0];
    p.trellis = reinterpret_cast<const uint32_t*>(trellis);
    p.suh = pre_rotated ? nullptr : reinterpret_cast<const __half*>(suh);
    p.svh = reinterpret_cast<const __half*>(svh);
    p.x = reinterpret_cast<const __half*>(x);
    p.x_stride = x_stride;
    p.xd = reinterpret_cast<uint32_t*>(scratch);
    p.sblk = cb == 2 ? reinterpret_cast<float*>(reinterpret_cast<char*>(scratch) + gv_xd_bytes(m, k)) : nullptr;
    p.acc = reinterpret_cast<float*>(state);
    p.acc_nb_stride = 16 * 128;
    p.out = out;
    p.out_stride = out_stride;
    p.out_rows = out_rows;
    p.out_scale = out_scale;
    p.k = k;
    p.n = n;
    p.m = m;
    return run_inline(a, K, cb, m, (flags >> 8) & 3, reinterpret_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// Small-M matmul that allocates nothing and takes no workspace.
//
// Some callers cannot allocate device memory at all: code running inside an
// allocator-less runtime (a custom serving loop that owns every byte of device
// memory up front, or a host thread that must not take the CUDA allocator's
// locks) still needs a matmul.  This entry point serves them: its scratch - the
// rotated activations and the split-K partial sums - lives in one file-scope
// device array below, reserved once per GPU when the library is loaded and held
// until the process exits.  Limits: m <= 16, k <= 32768, n <= 32768.
//
// The array is shared by every call on a device and keeps the last call's data,
// so calls that overlap on the GPU (different streams, or different host
// threads) race and corrupt each other's results; serialise them.  Each call
// clears the partial sums it will use before its kernels run.  The first call on
// each device looks up the array's device address (cudaGetSymbolAddress, with
// that device current).  With CUDA's lazy module loading that lookup is also what
// loads this library's device code on the device, reserving the array, so the
// caller makes one warm-up call per device before entering code that must not
// allocate, and before capturing a stream.
// ---------------------------------------------------------------------------
namespace exl3b200 {

constexpr int kNoAllocMaxM = 16;
constexpr int kNoAllocMaxK = 32768;
constexpr int kNoAllocMaxN = 32768;
constexpr size_t kNoAllocStateBytes = (size_t) (kNoAllocMaxN / 128) * 16 * 128 * sizeof(float);
constexpr size_t kNoAllocScratchBytes = (size_t) kNoAllocMaxM * kNoAllocMaxK * sizeof(uint32_t) +
                                        (size_t) kNoAllocMaxM * (kNoAllocMaxK / 128) * sizeof(float);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocStateBytes + kNoAllocScratchBytes];

static int noalloc_base(char** base)
{
    // one slot per device; threads that race on the first lookup store the same address
    static std::atomic<void*> cache[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kErrLaunch;
    void* p = cache[dev].load(std::memory_order_relaxed);
    if (!p) {
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return kErrLaunch;
        cache[dev].store(p, std::memory_order_relaxed);
    }
    *base = reinterpret_cast<char*>(p);
    return kOk;
}

}  // namespace exl3b200

extern "C" int exl3b200_gemv_noalloc(const void* x, long long x_stride, int m, int k, const void* trellis, int n,
                                     int K, int cb, const void* suh, const void* svh, void* out,
                                     long long out_stride, int out_dtype, void* stream)
{
    if (!x || !out || !suh) return kErrNullPointer;
    int rc = check_linear_args(trellis, svh, m, k, n, K, cb);
    if (rc != kOk) return rc;
    if (m > kNoAllocMaxM || k > kNoAllocMaxK || n > kNoAllocMaxN) return kErrBadShape;
    if (out_dtype < 0 || out_dtype > 2) return kErrBadArgument;
    if (x_stride < k || out_stride < n) return kErrBadShape;
    if (((uintptr_t) x & 3) || (x_stride & 1)) return kErrUnaligned;
    char* base = nullptr;
    rc = noalloc_base(&base);
    if (rc != kOk) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const size_t used_state = gv_state_bytes_per_problem(n);
    if (cudaMemsetAsync(base, 0, used_state, st) != cudaSuccess) return kErrLaunch;

    GvArgs a = {};
    a.nprob = 1;
    a.out_dtype = out_dtype;
    a.epi_mode = kEpiStore;
    GvProblem& p = a.inl[0];
    p.trellis = reinterpret_cast<const uint32_t*>(trellis);
    p.suh = reinterpret_cast<const __half*>(suh);
    p.svh = reinterpret_cast<const __half*>(svh);
    p.x = reinterpret_cast<const __half*>(x);
    p.x_stride = x_stride;
    char* scratch = base + kNoAllocStateBytes;
    p.xd = reinterpret_cast<uint32_t*>(scratch);
    p.sblk = cb == 2 ? reinterpret_cast<float*>(scratch + (size_t) kNoAllocMaxM * kNoAllocMaxK * sizeof(uint32_t))
                     : nullptr;
    p.acc = reinterpret_cast<float*>(base);
    p.acc_nb_stride = 16 * 128;
    p.out = out;
    p.out_stride = out_stride;
    p.k = k;
    p.n = n;
    p.m = m;
    return run_inline(a, K, cb, m, 0, st);
}
