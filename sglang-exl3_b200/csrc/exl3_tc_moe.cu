// Routed MoE on the tensor-core GEMM, for batches whose experts receive many rows
// each (speculative verify of 5 tokens per sequence, prefill, large decode
// batches).  The small-M pipeline (exl3_moe.cu) streams an expert's codes once per
// 16 rows; here every expert's codes are decoded once per 256 rows, into tcgen05
// MMAs.  Replaces the reference's large-M expert path: the per-expert Python loop
// over exl3_fat_gemm / exl3_fat_gemm_scatter (src/sglang_exl3/exl3.py:1154-1231,
// csrc/exl3_fat_gemm.cu:65-305), which synchronises on the host for the counts.
// Everything here stays on the device and is chained by programmatic dependent
// launch:
//
//   route kernel (1 CTA): groups the (token, slot) pairs by local expert (invalid
//     ids - negative or not local - are skipped, the reference's weight-0
//     sentinel, exl3.py:494-509); an expert's rows get consecutive slots (token and
//     weight lists) and an 8-aligned range of rows in the input images; writes the
//     problem tables (gate and up per active expert, then down), the problem of
//     every 256 x 256 output tile and the tile counts.
//   input stage:  H128(x[token] * suh) / sqrt(128) of every slot for gate and for
//     up, written into k-chunk-major swizzled images (the MMA's shared-memory
//     layout, so the GEMM copies each expert's rows with one bulk copy per k
//     chunk); zeroes the fp32 gate/up outputs and, unless accumulating, out.
//   grouped GEMM over gate and up.  When both have the same K (every checkpoint
//     seen), one launch whose 128-row tiles hold gate block j and up block j of an
//     expert side by side, with the clipped SwiGLU, its fp16 rounding, the down
//     projection's x * suh and H128 in the epilogue, written straight into the down
//     projection's image.  Otherwise two launches into fp32 rows and a SwiGLU stage
//     doing the same arithmetic (that of the small-M SwiGLU epilogue).
//   grouped GEMM: down, combined as out[token] += weight * y (fp32 vector atomics).
#include <algorithm>

#include "exl3_common.cuh"
#include "exl3_capi_internal.h"
#include "exl3_tc_internal.h"

namespace exl3b200 {

constexpr int kTmThreads = 1024;
constexpr int kTmMaxExperts = 2048;
constexpr int kTmMaxPairs = 65536;  // (token, slot) pairs of one launch (workspace sizing)
constexpr int kTmEpt = kTmMaxExperts / kTmThreads;  // experts per routing thread

static inline size_t tm_al(size_t v) { return (v + 255) & ~(size_t) 255; }

// tot[]: 0 gate+up tiles (fused: gate|up tiles), 1 gate tiles (= up tiles), 2 first up
//        tile, 3 down tiles, 4 routed slots, 5 zero
struct TmLayout {
    size_t tot, slot_token, slot_weight, slot_row, slot_exp, probs_gu, probs_d, tiles_gu, tiles_d;
    size_t xt_g, xt_u, xt_d, gu_out, bytes;
    long long xt_rows;
    int act_max, mt_max;
};

static TmLayout tm_layout(int pmax, int experts, int hidden, int inter)
{
    TmLayout L;
    L.act_max = std::min(experts, pmax);                // experts that can receive a row
    // every expert's rows rounded up to 8; each k-chunk slab a whole number of 8-row groups
    L.xt_rows = ((long long) pmax + 7ll * L.act_max + 7) & ~7ll;
    L.mt_max = pmax / 256 + L.act_max;                  // sum over experts of ceil(rows / 256)
    const long long ntg = (inter + 255) / 256, ntd = (hidden + 255) / 256;
    // fused gate|up tiles: inter / 128 blocks x sum over experts of ceil(rows / 96)
    const long long fused_tiles = (long long) (inter / 128) * (pmax / kTcSwRows + L.act_max);
    size_t o = 0;
    L.tot = o; o = tm_al(o + 16 * sizeof(int));
    L.slot_token = o; o = tm_al(o + (size_t) pmax * sizeof(int));
    L.slot_weight = o; o = tm_al(o + (size_t) pmax * sizeof(float));
    L.slot_row = o; o = tm_al(o + (size_t) pmax * sizeof(int));
    L.slot_exp = o; o = tm_al(o + (size_t) pmax * sizeof(int));
    L.probs_gu = o; o = tm_al(o + (size_t) 2 * L.act_max * sizeof(TcProblem));
    L.probs_d = o; o = tm_al(o + (size_t) L.act_max * sizeof(TcProblem));
    L.tiles_gu = o; o = tm_al(o + (size_t) std::max(2 * ntg * L.mt_max, fused_tiles) * sizeof(int));
    L.tiles_d = o; o = tm_al(o + (size_t) ntd * L.mt_max * sizeof(int));
    L.xt_g = o; o = tm_al(o + (size_t) L.xt_rows * hidden * 2);
    L.xt_u = o; o = tm_al(o + (size_t) L.xt_rows * hidden * 2);
    L.xt_d = o; o = tm_al(o + (size_t) L.xt_rows * inter * 2);
    L.gu_out = o; o = tm_al(o + (size_t) pmax * 2 * inter * sizeof(float));
    L.bytes = o;
    return L;
}

struct TmArgs {
    const int* ids;
    const float* weights;
    const long long *gt, *gu, *gv, *ut, *uu, *uv, *dt, *du, *dv;
    const __half* x;
    long long x_stride;
    float* out;
    long long out_stride;
    char* scratch;
    TmLayout L;
    int tokens, topk, experts, hidden, inter, accumulate;
    int fused;  // gate and up in one launch with the SwiGLU epilogue (same K)
    float swiglu_limit;
};

__device__ __forceinline__ int* tm_tot(const TmArgs& t) { return reinterpret_cast<int*>(t.scratch + t.L.tot); }

// Inclusive block-wide scan of NV values per thread over kTmThreads threads.
template <int NV>
__device__ __forceinline__ void tm_block_scan(int (&v)[NV], int (*s_warp)[NV])
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
        for (int j = 0; j < NV; ++j) {
            const int n = __shfl_up_sync(0xffffffffu, v[j], o);
            if (lane >= o) v[j] += n;
        }
    }
    if (lane == 31)
#pragma unroll
        for (int j = 0; j < NV; ++j) s_warp[warp][j] = v[j];
    __syncthreads();
    if (warp == 0) {
        int w[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) w[j] = s_warp[lane][j];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
#pragma unroll
            for (int j = 0; j < NV; ++j) {
                const int n = __shfl_up_sync(0xffffffffu, w[j], o);
                if (lane >= o) w[j] += n;
            }
        }
#pragma unroll
        for (int j = 0; j < NV; ++j) s_warp[lane][j] = w[j];  // inclusive over warps
    }
    __syncthreads();
    if (warp > 0)
#pragma unroll
        for (int j = 0; j < NV; ++j) v[j] += s_warp[warp - 1][j];
}

__global__ __launch_bounds__(kTmThreads) void exl3_tm_route_kernel(const TmArgs t)
{
    __shared__ int s_count[kTmMaxExperts];
    __shared__ int s_slot[kTmMaxExperts];  // first slot of each expert
    __shared__ int s_row[kTmMaxExperts];   // first image row of each expert
    __shared__ int s_fill[kTmMaxExperts];  // rows placed so far (second pass)
    __shared__ int s_warp[32][5];

    const int tid = threadIdx.x;
    const TmLayout& L = t.L;
    const int P = t.tokens * t.topk;
    for (int e = tid; e < kTmMaxExperts; e += kTmThreads) s_count[e] = 0;
    __syncthreads();
    for (int p = tid; p < P; p += kTmThreads) {
        const int e = t.ids[p];
        if (e >= 0 && e < t.experts) atomicAdd(&s_count[e], 1);
    }
    for (int e = tid; e < kTmMaxExperts; e += kTmThreads) s_fill[e] = 0;
    __syncthreads();

    // per expert: rows, rows rounded up to 8, active (0/1), 256-row tiles, fused-tile rows
    int c[kTmEpt], ex[kTmEpt][5], sum[5] = {0, 0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < kTmEpt; ++j) {
        c[j] = s_count[tid * kTmEpt + j];
        const int v[5] = {c[j], (c[j] + 7) & ~7, c[j] > 0 ? 1 : 0, (c[j] + 255) / 256,
                          (c[j] + kTcSwRows - 1) / kTcSwRows};
#pragma unroll
        for (int q = 0; q < 5; ++q) {
            ex[j][q] = sum[q];
            sum[q] += v[q];
        }
    }
    int inc[5] = {sum[0], sum[1], sum[2], sum[3], sum[4]};
    tm_block_scan<5>(inc, s_warp);
    int base[5];
#pragma unroll
    for (int q = 0; q < 5; ++q) base[q] = inc[q] - sum[q];
#pragma unroll
    for (int j = 0; j < kTmEpt; ++j) {
        s_slot[tid * kTmEpt + j] = base[0] + ex[j][0];
        s_row[tid * kTmEpt + j] = base[1] + ex[j][1];
    }
    __syncthreads();
    const int total_rows = s_warp[31][0];
    const int total_mt = s_warp[31][3];
    const int total_mtf = s_warp[31][4];

    int* slot_token = reinterpret_cast<int*>(t.scratch + L.slot_token);
    float* slot_weight = reinterpret_cast<float*>(t.scratch + L.slot_weight);
    int* slot_row = reinterpret_cast<int*>(t.scratch + L.slot_row);
    int* slot_exp = reinterpret_cast<int*>(t.scratch + L.slot_exp);
    // a pair's place among its expert's rows from a second count (the order within an
    // expert is arbitrary; rows are independent): no per-pair state limits the pairs
    for (int p = tid; p < P; p += kTmThreads) {
        const int e = t.ids[p];
        if (e < 0 || e >= t.experts) continue;
        const int rank = atomicAdd(&s_fill[e], 1);
        const int s = s_slot[e] + rank;
        slot_token[s] = p / t.topk;
        slot_weight[s] = t.weights[p];
        slot_row[s] = s_row[e] + rank;
        slot_exp[s] = e;
    }

    // problems and tile lists: gate tiles of every expert, then up tiles, then (own
    // list) down tiles; within a problem the 256-row tiles run fastest
    const int H = t.hidden, I = t.inter;
    const int ntg = (I + 255) / 256, ntd = (H + 255) / 256, ntf = I / 128;
    const int G = ntg * total_mt;
    TcProblem* pg = reinterpret_cast<TcProblem*>(t.scratch + L.probs_gu);
    TcProblem* pd = reinterpret_cast<TcProblem*>(t.scratch + L.probs_d);
    int* tg = reinterpret_cast<int*>(t.scratch + L.tiles_gu);
    int* td = reinterpret_cast<int*>(t.scratch + L.tiles_d);
    float* gu_out = reinterpret_cast<float*>(t.scratch + L.gu_out);
#pragma unroll
    for (int j = 0; j < kTmEpt; ++j) {
        const int e = tid * kTmEpt + j;
        if (c[j] == 0) continue;
        const int a = base[2] + ex[j][2];    // active-expert index
        const int mtp = base[3] + ex[j][3];  // 256-row tiles before this expert
        const int mt = (c[j] + 255) / 256;
        const int mtpf = base[4] + ex[j][4];  // fused tiles' row groups before this expert
        const int mtf = (c[j] + kTcSwRows - 1) / kTcSwRows;
        TcProblem g = {};
        g.m = c[j];
        g.mtiles = mt;
        g.row0 = s_row[e];
        g.slot0 = s_slot[e];
        TcProblem u = g, d = g;
        g.xt = reinterpret_cast<const uint8_t*>(t.scratch + L.xt_g);
        u.xt = reinterpret_cast<const uint8_t*>(t.scratch + L.xt_u);
        d.xt = reinterpret_cast<const uint8_t*>(t.scratch + L.xt_d);
        g.trellis = reinterpret_cast<const uint8_t*>(t.gt[e]);
        g.svh = reinterpret_cast<const __half*>(t.gv[e]);
        g.out = gu_out + (size_t) s_slot[e] * 2 * I;
        g.tile_begin = ntg * mtp;
        u.trellis = reinterpret_cast<const uint8_t*>(t.ut[e]);
        u.svh = reinterpret_cast<const __half*>(t.uv[e]);
        u.out = g.out + I;
        u.tile_begin = G + ntg * mtp;
        d.trellis = reinterpret_cast<const uint8_t*>(t.dt[e]);
        d.svh = reinterpret_cast<const __half*>(t.dv[e]);
        d.out = nullptr;
        d.tile_begin = ntd * mtp;
        if (t.fused) {
            // one problem (gate, up = the next entry) in 96-row tiles, no fp32 rows
            g.mtiles = mtf;
            g.tile_begin = ntf * mtpf;
            g.out = nullptr;
            g.suh2 = reinterpret_cast<const __half*>(t.du[e]);
            u.out = nullptr;
            for (int i = 0; i < ntf * mtf; ++i) tg[g.tile_begin + i] = 2 * a;
        } else {
            for (int i = 0; i < ntg * mt; ++i) {
                tg[g.tile_begin + i] = 2 * a;
                tg[u.tile_begin + i] = 2 * a + 1;
            }
        }
        pg[2 * a] = g;
        pg[2 * a + 1] = u;
        pd[a] = d;
        for (int i = 0; i < ntd * mt; ++i) td[d.tile_begin + i] = a;
    }
    if (tid == 0) {
        int* tot = tm_tot(t);
        tot[0] = t.fused ? ntf * total_mtf : 2 * G;
        tot[1] = G;
        tot[2] = G;
        tot[3] = ntd * total_mt;
        tot[4] = total_rows;
        tot[5] = 0;
    }
}

// One warp per (slot, 128-block): the row block of x[token] loaded once, rotated
// with the gate's and with the up projection's suh (rotate_block's roundings) into
// the two images; the grid also zeroes the fp32 gate/up rows and (unless
// accumulating) out.
__global__ __launch_bounds__(256) void exl3_tm_input_kernel(const TmArgs t)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const TmLayout& L = t.L;
    const int lane = threadIdx.x & 31;
    const int H = t.hidden, I = t.inter;
    const int nblk = H >> 7;
    const int rows = tm_tot(t)[4];
    const int tasks = rows * nblk;
    const int* slot_token = reinterpret_cast<const int*>(t.scratch + L.slot_token);
    const int* slot_row = reinterpret_cast<const int*>(t.scratch + L.slot_row);
    const int* slot_exp = reinterpret_cast<const int*>(t.scratch + L.slot_exp);
    const int warps = gridDim.x * (blockDim.x >> 5);
    const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    for (int task = gw; task < tasks; task += warps) {
        const int s = task / nblk, b = task - s * nblk;
        const int e = slot_exp[s];
        const int row = slot_row[s];
        const __half* src = t.x + (size_t) slot_token[s] * t.x_stride + b * 128;
        float xv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) xv[i] = __half2float(src[lane + 32 * i]);
#pragma unroll
        for (int which = 0; which < 2; ++which) {
            const __half* suh = reinterpret_cast<const __half*>(which ? t.uu[e] : t.gu[e]) + b * 128;
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                v[i] = __half2float(__float2half_rn(__fmul_rn(xv[i], __half2float(suh[lane + 32 * i]))));
            warp_fwht128(v, lane);
            uint8_t* img = reinterpret_cast<uint8_t*>(t.scratch + (which ? L.xt_u : L.xt_g));
#pragma unroll
            for (int i = 0; i < 4; ++i)
                *reinterpret_cast<__half*>(img + tc_image_offset(L.xt_rows, row, b * 128 + lane + 32 * i)) =
                    __float2half_rn(__fmul_rn(v[i], kHadScale));
        }
    }
    // zero the gate/up rows (split tiles add into them; not used when fused) and the output
    const int gthreads = gridDim.x * blockDim.x;
    const int gt = blockIdx.x * blockDim.x + threadIdx.x;
    float4* gu4 = reinterpret_cast<float4*>(t.scratch + L.gu_out);
    const long long n_gu4 = t.fused ? 0 : (long long) rows * 2 * I / 4;
    for (long long i = gt; i < n_gu4; i += gthreads) gu4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!t.accumulate) {
        const long long n_out = (long long) t.tokens * H;
        for (long long i = gt; i < n_out; i += gthreads) {
            const long long r = i / H, col = i - r * H;
            t.out[r * t.out_stride + col] = 0.f;
        }
    }
}

// One warp per (slot, 128-block of the intermediate): clipped SwiGLU of the gate
// and up rows, fp16, then H128(act * suh_down) / sqrt(128) into the down image
// (the arithmetic of the small-M MoE's SwiGLU epilogue, exl3_epilogue.cuh).
__global__ __launch_bounds__(256) void exl3_tm_swiglu_kernel(const TmArgs t)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const TmLayout& L = t.L;
    const int lane = threadIdx.x & 31;
    const int I = t.inter;
    const int nblk = I >> 7;
    const int rows = tm_tot(t)[4];
    const int tasks = rows * nblk;
    const int* slot_row = reinterpret_cast<const int*>(t.scratch + L.slot_row);
    const int* slot_exp = reinterpret_cast<const int*>(t.scratch + L.slot_exp);
    const float* gu_out = reinterpret_cast<const float*>(t.scratch + L.gu_out);
    uint8_t* img = reinterpret_cast<uint8_t*>(t.scratch + L.xt_d);
    const float lim = t.swiglu_limit;
    const bool clip = lim > 0.f && lim < 3.0e38f;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < tasks; task += warps) {
        const int s = task / nblk, b = task - s * nblk;
        const float* g = gu_out + (size_t) s * 2 * I + b * 128;
        const float* u = g + I;
        const __half* suh = reinterpret_cast<const __half*>(t.du[slot_exp[s]]) + b * 128;
        float act[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float gv = __ldcg(g + lane + 32 * i), uv = __ldcg(u + lane + 32 * i);
            if (clip) {
                gv = fminf(gv, lim);
                uv = fminf(fmaxf(uv, -lim), lim);
            }
            const float sg = gv / (1.0f + expf(-gv));
            act[i] = __half2float(__float2half_rn(sg * uv));
            act[i] = __half2float(__float2half_rn(__fmul_rn(act[i], __half2float(suh[lane + 32 * i]))));
        }
        warp_fwht128(act, lane);
        const int row = slot_row[s];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            *reinterpret_cast<__half*>(img + tc_image_offset(L.xt_rows, row, b * 128 + lane + 32 * i)) =
                __float2half_rn(__fmul_rn(act[i], kHadScale));
    }
}

static int tm_launch(const void* kern, int grid, int block, bool pdl, cudaStream_t st, void** args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) std::max(grid, 1));
    cfg.blockDim = dim3((unsigned) block);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, kern, args) == cudaSuccess ? kOk : kErrLaunch;
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" size_t exl3b200_moe_tc_scratch_size(int max_tokens, int topk, int num_experts, int hidden, int inter)
{
    if (max_tokens < 1 || topk < 1 || num_experts < 1 || num_experts > kTmMaxExperts) return 0;
    if (hidden <= 0 || inter <= 0 || hidden % 128 || inter % 128 || (long long) max_tokens * topk > kTmMaxPairs)
        return 0;
    return tm_layout(max_tokens * topk, num_experts, hidden, inter).bytes;
}

extern "C" int exl3b200_moe_tc(const void* x, long long x_stride, int tokens, int hidden, int inter,
                               const int* topk_ids, const float* topk_weights, int topk, int num_experts,
                               const long long* gate_trellis, const long long* gate_suh, const long long* gate_svh,
                               const long long* up_trellis, const long long* up_suh, const long long* up_svh,
                               const long long* down_trellis, const long long* down_suh, const long long* down_svh,
                               int K_gate, int K_up, int K_down, int cb, float swiglu_limit, float* out,
                               long long out_stride, int accumulate, int max_tokens, void* scratch,
                               size_t scratch_bytes, void* stream)
{
    if (!x || !topk_ids || !topk_weights || !out || !scratch) return kErrNullPointer;
    if (!gate_trellis || !gate_suh || !gate_svh || !up_trellis || !up_suh || !up_svh || !down_trellis ||
        !down_suh || !down_svh)
        return kErrNullPointer;
    if (tokens < 1 || tokens > max_tokens || topk < 1 || (long long) max_tokens * topk > kTmMaxPairs)
        return kErrBadShape;
    if (num_experts < 1 || num_experts > kTmMaxExperts) return kErrBadShape;
    if (hidden <= 0 || inter <= 0 || hidden % 128 || inter % 128 || x_stride < hidden || out_stride < hidden)
        return kErrBadShape;
    for (int Kx : {K_gate, K_up, K_down})
        if (Kx < 2 || Kx > 4) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (((uintptr_t) scratch & 255) || ((uintptr_t) x & 1) || ((uintptr_t) out & 15) || (out_stride & 3))
        return kErrUnaligned;
    const TmLayout L = tm_layout(max_tokens * topk, num_experts, hidden, inter);
    if (scratch_bytes < L.bytes) return kErrWorkspace;

    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char* sc = reinterpret_cast<char*>(scratch);
    TmArgs t;
    t.ids = topk_ids;
    t.weights = topk_weights;
    t.gt = gate_trellis; t.gu = gate_suh; t.gv = gate_svh;
    t.ut = up_trellis; t.uu = up_suh; t.uv = up_svh;
    t.dt = down_trellis; t.du = down_suh; t.dv = down_svh;
    t.x = reinterpret_cast<const __half*>(x);
    t.x_stride = x_stride;
    t.out = out;
    t.out_stride = out_stride;
    t.scratch = sc;
    t.L = L;
    t.tokens = tokens;
    t.topk = topk;
    t.experts = num_experts;
    t.hidden = hidden;
    t.inter = inter;
    t.accumulate = accumulate;
    t.fused = K_gate == K_up ? 1 : 0;
    t.swiglu_limit = swiglu_limit;
    void* args[] = {&t};

    int rc = tm_launch((const void*) exl3_tm_route_kernel, 1, kTmThreads, false, st, args);
    if (rc != kOk) return rc;
    const int sms = tc_device_sms();
    const int pairs = tokens * topk;
    const int in_grid = std::min((pairs * (hidden / 128) + 7) / 8, 8 * sms);
    rc = tm_launch((const void*) exl3_tm_input_kernel, in_grid, 256, true, st, args);
    if (rc != kOk) return rc;

    const int* tot = reinterpret_cast<const int*>(sc + L.tot);
    TcGroupedCall g = {};
    g.xt_rows = L.xt_rows;
    g.probs = reinterpret_cast<const TcProblem*>(sc + L.probs_gu);
    g.tile_prob = reinterpret_cast<const int*>(sc + L.tiles_gu);
    g.k = hidden;
    g.n = inter;
    g.out = reinterpret_cast<float*>(sc + L.gu_out);  // rows come from the problems
    g.out_stride = 2 * inter;
    g.mode = kTcGroupedStore;
    if (t.fused) {
        // one launch over the gate|up tiles; its epilogue writes the down image
        g.mode = kTcGroupedSwiglu;
        g.out = nullptr;
        g.out_stride = 0;
        g.img = reinterpret_cast<uint8_t*>(sc + L.xt_d);
        g.swiglu_limit = swiglu_limit;
        g.dev_tiles = tot + 0;
        g.dev_tile_base = tot + 5;
        rc = tc_grouped_matmul(g, K_gate, cb, st);
    } else {
        g.dev_tiles = tot + 1;  // gate tiles: [0, G)
        g.dev_tile_base = tot + 5;
        rc = tc_grouped_matmul(g, K_gate, cb, st);
        if (rc != kOk) return rc;
        g.dev_tile_base = tot + 2;  // up tiles: [G, 2G)
        rc = tc_grouped_matmul(g, K_up, cb, st);
    }
    if (rc != kOk) return rc;

    if (!t.fused) {
        const int sw_grid = std::min((pairs * (inter / 128) + 7) / 8, 8 * sms);
        rc = tm_launch((const void*) exl3_tm_swiglu_kernel, sw_grid, 256, true, st, args);
        if (rc != kOk) return rc;
    }

    TcGroupedCall d = {};
    d.xt_rows = L.xt_rows;
    d.probs = reinterpret_cast<const TcProblem*>(sc + L.probs_d);
    d.tile_prob = reinterpret_cast<const int*>(sc + L.tiles_d);
    d.dev_tiles = tot + 3;
    d.dev_tile_base = nullptr;
    d.k = inter;
    d.n = hidden;
    d.out = out;
    d.out_stride = out_stride;
    d.slot_token = reinterpret_cast<const int*>(sc + L.slot_token);
    d.slot_weight = reinterpret_cast<const float*>(sc + L.slot_weight);
    d.mode = kTcGroupedCombine;
    return tc_grouped_matmul(d, K_down, cb, st);
}

// ---------------------------------------------------------------------------
// One routed linear on the tensor cores: out[out_rows[r]] += out_scale[r] * (x[r] @ W)
// for any m (the large-M form of the reference's exl3_fat_gemm_scatter).  A setup
// kernel writes the rotated input image, the row and weight lists and a one-problem
// table; then one grouped launch in combine mode.
// ---------------------------------------------------------------------------
namespace exl3b200 {

struct GcLayout {
    size_t tot, prob, tiles, token, weight, img, bytes;
    long long xt_rows;
    int mtiles, ntiles;
};

static GcLayout gc_layout(int m, int k, int n)
{
    GcLayout L;
    L.xt_rows = ((long long) m + 7) & ~7ll;
    L.mtiles = (m + 255) / 256;
    L.ntiles = (n + 255) / 256;
    size_t o = 0;
    L.tot = o; o = tm_al(o + 16 * sizeof(int));
    L.prob = o; o = tm_al(o + sizeof(TcProblem));
    L.tiles = o; o = tm_al(o + (size_t) L.mtiles * L.ntiles * sizeof(int));
    L.token = o; o = tm_al(o + (size_t) m * sizeof(int));
    L.weight = o; o = tm_al(o + (size_t) m * sizeof(float));
    L.img = o; o = tm_al(o + (size_t) L.xt_rows * k * 2);
    L.bytes = o;
    return L;
}

struct GcArgs {
    const __half* x;
    long long x_stride;
    const __half* suh;  // null: x is already rotated
    const int* rows;    // null: row r
    const float* scale; // null: 1
    const uint8_t* trellis;
    const __half* svh;
    char* scratch;
    GcLayout L;
    int m, k;
};

__global__ __launch_bounds__(256) void exl3_gc_setup_kernel(const GcArgs g)
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const GcLayout& L = g.L;
    const int tid = blockIdx.x * blockDim.x + threadIdx.x;
    const int nth = gridDim.x * blockDim.x;
    if (tid == 0) {
        TcProblem p = {};
        p.xt = reinterpret_cast<const uint8_t*>(g.scratch + L.img);
        p.trellis = g.trellis;
        p.svh = g.svh;
        p.m = g.m;
        p.mtiles = L.mtiles;
        *reinterpret_cast<TcProblem*>(g.scratch + L.prob) = p;
        reinterpret_cast<int*>(g.scratch + L.tot)[0] = L.mtiles * L.ntiles;
    }
    int* tiles = reinterpret_cast<int*>(g.scratch + L.tiles);
    for (int i = tid; i < L.mtiles * L.ntiles; i += nth) tiles[i] = 0;
    int* token = reinterpret_cast<int*>(g.scratch + L.token);
    float* weight = reinterpret_cast<float*>(g.scratch + L.weight);
    for (int r = tid; r < g.m; r += nth) {
        token[r] = g.rows ? g.rows[r] : r;
        weight[r] = g.scale ? g.scale[r] : 1.f;
    }
    const int lane = threadIdx.x & 31;
    const int nblk = g.k >> 7;
    uint8_t* img = reinterpret_cast<uint8_t*>(g.scratch + L.img);
    const int warps = nth >> 5;
    for (int task = tid >> 5; task < g.m * nblk; task += warps) {
        const int r = task / nblk, b = task - r * nblk;
        __half h[4];
        rotate_block(g.x + (size_t) r * g.x_stride + b * 128, g.suh ? g.suh + b * 128 : nullptr, lane, h);
#pragma unroll
        for (int i = 0; i < 4; ++i)
            *reinterpret_cast<__half*>(img + tc_image_offset(L.xt_rows, r, b * 128 + lane + 32 * i)) = h[i];
    }
}

}  // namespace exl3b200

extern "C" size_t exl3b200_gemm_combine_scratch_size(int m, int k, int n)
{
    if (m < 1 || k <= 0 || n <= 0 || k % 128 || n % 128) return 0;
    return gc_layout(m, k, n).bytes;
}

extern "C" int exl3b200_gemm_combine(const void* x, long long x_stride, int m, int k, const void* trellis, int n,
                                     int K, int cb, const void* suh, const void* svh, float* out,
                                     long long out_stride, const int* out_rows, const float* out_scale, int flags,
                                     void* scratch, size_t scratch_bytes, void* stream)
{
    if (!x || !trellis || !svh || !out || !scratch) return kErrNullPointer;
    if (K < 2 || K > 4) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (m < 1 || k <= 0 || n <= 0 || k % 128 || n % 128 || x_stride < k || out_stride < n) return kErrBadShape;
    const bool pre_rotated = (flags & EXL3B200_FLAG_INPUT_ROTATED) != 0;
    if (!pre_rotated && !suh) return kErrNullPointer;
    if (((uintptr_t) x & 1) || ((uintptr_t) trellis & 15) || ((uintptr_t) svh & 15) || ((uintptr_t) scratch & 255) ||
        ((uintptr_t) out & 15) || (out_stride & 3))
        return kErrUnaligned;
    const GcLayout L = gc_layout(m, k, n);
    if (scratch_bytes < L.bytes) return kErrWorkspace;
    if ((long long) L.mtiles * L.ntiles > 0x7fffffffLL) return kErrBadShape;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char* sc = reinterpret_cast<char*>(scratch);
    GcArgs g;
    g.x = reinterpret_cast<const __half*>(x);
    g.x_stride = x_stride;
    g.suh = pre_rotated ? nullptr : reinterpret_cast<const __half*>(suh);
    g.rows = out_rows;
    g.scale = out_scale;
    g.trellis = reinterpret_cast<const uint8_t*>(trellis);
    g.svh = reinterpret_cast<const __half*>(svh);
    g.scratch = sc;
    g.L = L;
    g.m = m;
    g.k = k;
    void* args[] = {&g};
    const int grid = std::min((m * (k / 128) + 7) / 8, 4 * tc_device_sms());
    int rc = tm_launch((const void*) exl3_gc_setup_kernel, grid, 256, true, st, args);
    if (rc != kOk) return rc;
    TcGroupedCall c = {};
    c.xt_rows = L.xt_rows;
    c.probs = reinterpret_cast<const TcProblem*>(sc + L.prob);
    c.tile_prob = reinterpret_cast<const int*>(sc + L.tiles);
    c.dev_tiles = reinterpret_cast<const int*>(sc + L.tot);
    c.dev_tile_base = nullptr;
    c.k = k;
    c.n = n;
    c.out = out;
    c.out_stride = out_stride;
    c.slot_token = reinterpret_cast<const int*>(sc + L.token);
    c.slot_weight = reinterpret_cast<const float*>(sc + L.weight);
    c.mode = kTcGroupedCombine;
    return tc_grouped_matmul(c, K, cb, st);
}
