// Routed-MoE and batched-expert EXL3 matmuls on the grouped small-M kernels.
//
// Replaces the reference's cooperative single-row fused MoE (csrc/p2b_moe.cu:14-468,
// driven once per token row by a Python loop, src/sglang_exl3/exl3.py:868-957) and
// its batched expert GEMV (csrc/p2b_batched.cu:13-101,
// src/sglang_exl3/exl3.py:960-1110).  Everything stays on the device:
//
//   route kernel (1 CTA): the (token, slot) pairs of the top-k routing are grouped
//     by local expert with shared-memory atomics (invalid ids - negative or not
//     local - are skipped, the reference's weight-0 sentinel, exl3.py:494-509);
//     each expert's rows form problems of at most 16 rows; the kernel writes the
//     (gate, up) and down problem tables, the per-row token and weight lists, the
//     task totals, and zeroes the fp32 output unless accumulating.
//   input stage:   rotated gate and up inputs of every row, H128(x[token] * suh_e)
//   matmul:        gate and up (one launch when both have the same K)
//   epilogue:      SwiGLU with the optional clip, then the rotated down input
//   matmul:        down (its input is already rotated)
//   epilogue:      y * routing weight added into out[token] (fp32)
//
// The kernels after the router are chained with programmatic dependent launch and
// read their extents from device memory, so a decode step of any batch and routing
// needs no host synchronisation and is CUDA-graph capturable.
#include <algorithm>

#include "exl3_common.cuh"
#include "exl3_capi_internal.h"
#include "exl3_grouped.cuh"

namespace exl3b200 {

constexpr int kRouteThreads = 1024;
constexpr int kMaxLocalExperts = 2048;
constexpr int kMaxPairs = 65536;  // (token, slot) pairs of one launch (workspace sizing)
constexpr int kExpertsPerThread = kMaxLocalExperts / kRouteThreads;

static inline size_t al256(size_t v) { return (v + 255) & ~(size_t) 255; }

struct MoeLayout {
    // scratch
    size_t tot, token, weight, tab_gu, tab_d, xd_g, xd_u, sb_g, sb_u, xd_d, sb_d, scratch_bytes;
    // state
    size_t acc_g, acc_u, acc_d, state_bytes;
};

static MoeLayout moe_layout(int pmax, int hidden, int inter)
{
    MoeLayout L;
    size_t o = 0;
    L.tot = o; o = al256(o + 16 * sizeof(int));
    L.token = o; o = al256(o + (size_t) pmax * sizeof(int));
    L.weight = o; o = al256(o + (size_t) pmax * sizeof(float));
    L.tab_gu = o; o = al256(o + (size_t) 2 * pmax * sizeof(GvProblem));
    L.tab_d = o; o = al256(o + (size_t) pmax * sizeof(GvProblem));
    L.xd_g = o; o = al256(o + (size_t) pmax * hidden * sizeof(uint32_t));
    L.xd_u = o; o = al256(o + (size_t) pmax * hidden * sizeof(uint32_t));
    L.sb_g = o; o = al256(o + (size_t) pmax * (hidden / 128) * sizeof(float));
    L.sb_u = o; o = al256(o + (size_t) pmax * (hidden / 128) * sizeof(float));
    L.xd_d = o; o = al256(o + (size_t) pmax * inter * sizeof(uint32_t));
    L.sb_d = o; o = al256(o + (size_t) pmax * (inter / 128) * sizeof(float));
    L.scratch_bytes = o;
    o = 0;
    L.acc_g = o; o = al256(o + (size_t) (inter / 128) * pmax * 128 * sizeof(float));
    L.acc_u = o; o = al256(o + (size_t) (inter / 128) * pmax * 128 * sizeof(float));
    L.acc_d = o; o = al256(o + (size_t) (hidden / 128) * pmax * 128 * sizeof(float));
    L.state_bytes = o;
    return L;
}

struct MoeTables {
    const int* ids;
    const float* weights;
    const long long *gt, *gu, *gv, *ut, *uu, *uv, *dt, *du, *dv;
    const __half* x;
    long long x_stride;
    float* out;
    long long out_stride;
    char* scratch;
    char* state;
    int tokens, topk, experts, hidden, inter, pmax, mul1, accumulate;
    int prob_rows;  // rows per grouped problem: 8 (one row group, 8 tiles per warp) or 16
};

__global__ __launch_bounds__(kRouteThreads) void exl3_moe_route_kernel(const MoeTables t, MoeLayout L)
{
    __shared__ int s_count[kMaxLocalExperts];
    __shared__ int s_slot[kMaxLocalExperts];   // exclusive prefix of rows
    __shared__ int s_prob[kMaxLocalExperts];   // exclusive prefix of problems
    __shared__ int s_fill[kMaxLocalExperts];   // rows placed so far (second pass)
    __shared__ int s_warp[32][2];

    const int tid = threadIdx.x;
    const int P = t.tokens * t.topk;
    for (int e = tid; e < t.experts; e += kRouteThreads) s_count[e] = 0;
    __syncthreads();
    for (int p = tid; p < P; p += kRouteThreads) {
        const int e = t.ids[p];
        if (e >= 0 && e < t.experts) atomicAdd(&s_count[e], 1);
    }
    __syncthreads();

    // exclusive scans over experts: rows and 16-row problems
    {
        constexpr int EPT = kExpertsPerThread;
        int rows[EPT], probs[EPT], rsum = 0, psum = 0;
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
            const int e = tid * EPT + j;
            const int c = e < t.experts ? s_count[e] : 0;
            rows[j] = rsum;
            probs[j] = psum;
            rsum += c;
            psum += (c + t.prob_rows - 1) / t.prob_rows;
        }
        const int lane = tid & 31, warp = tid >> 5;
        int ri = rsum, pi = psum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int rn = __shfl_up_sync(0xffffffffu, ri, o);
            const int pn = __shfl_up_sync(0xffffffffu, pi, o);
            if (lane >= o) {
                ri += rn;
                pi += pn;
            }
        }
        if (lane == 31) {
            s_warp[warp][0] = ri;
            s_warp[warp][1] = pi;
        }
        __syncthreads();
        if (warp == 0) {
            int wr = s_warp[lane][0], wp = s_warp[lane][1];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int rn = __shfl_up_sync(0xffffffffu, wr, o);
                const int pn = __shfl_up_sync(0xffffffffu, wp, o);
                if (lane >= o) {
                    wr += rn;
                    wp += pn;
                }
            }
            s_warp[lane][0] = wr;  // inclusive
            s_warp[lane][1] = wp;
        }
        __syncthreads();
        const int rbase = (warp ? s_warp[warp - 1][0] : 0) + ri - rsum;
        const int pbase = (warp ? s_warp[warp - 1][1] : 0) + pi - psum;
#pragma unroll
        for (int j = 0; j < EPT; ++j) {
            const int e = tid * EPT + j;
            if (e < t.experts) {
                s_slot[e] = rbase + rows[j];
                s_prob[e] = pbase + probs[j];
            }
        }
    }
    __syncthreads();
    const int total_rows = s_warp[31][0];
    const int total_probs = s_warp[31][1];

    // second pass: a pair's place among its expert's rows from a second count (the
    // order within an expert is arbitrary; rows are independent), so no per-pair state
    // limits the pairs of a launch
    for (int e = tid; e < t.experts; e += kRouteThreads) s_fill[e] = 0;
    __syncthreads();
    int* token = reinterpret_cast<int*>(t.scratch + L.token);
    float* weight = reinterpret_cast<float*>(t.scratch + L.weight);
    for (int p = tid; p < P; p += kRouteThreads) {
        const int e = t.ids[p];
        if (e < 0 || e >= t.experts) continue;
        const int slot = s_slot[e] + atomicAdd(&s_fill[e], 1);
        token[slot] = p / t.topk;
        weight[slot] = t.weights[p];
    }

    GvProblem* gu = reinterpret_cast<GvProblem*>(t.scratch + L.tab_gu);
    GvProblem* dn = reinterpret_cast<GvProblem*>(t.scratch + L.tab_d);
    const int H = t.hidden, I = t.inter, pmax = t.pmax;
    for (int e = tid; e < t.experts; e += kRouteThreads) {
        const int c = s_count[e];
        for (int j = 0; j * t.prob_rows < c; ++j) {
            const int q = s_prob[e] + j;
            const int first = s_slot[e] + j * t.prob_rows;
            const int m = min(t.prob_rows, c - j * t.prob_rows);
            GvProblem g = {};
            g.k = H;
            g.n = I;
            g.m = m;
            g.x = t.x;
            g.x_stride = t.x_stride;
            g.x_rows = token + first;
            g.acc_nb_stride = pmax * 128;
            GvProblem u = g;
            g.trellis = reinterpret_cast<const uint32_t*>(t.gt[e]);
            g.suh = reinterpret_cast<const __half*>(t.gu[e]);
            g.svh = reinterpret_cast<const __half*>(t.gv[e]);
            u.trellis = reinterpret_cast<const uint32_t*>(t.ut[e]);
            u.suh = reinterpret_cast<const __half*>(t.uu[e]);
            u.svh = reinterpret_cast<const __half*>(t.uv[e]);
            g.xd = reinterpret_cast<uint32_t*>(t.scratch + L.xd_g) + (size_t) first * H;
            u.xd = reinterpret_cast<uint32_t*>(t.scratch + L.xd_u) + (size_t) first * H;
            g.sblk = t.mul1 ? reinterpret_cast<float*>(t.scratch + L.sb_g) + (size_t) first * (H / 128) : nullptr;
            u.sblk = t.mul1 ? reinterpret_cast<float*>(t.scratch + L.sb_u) + (size_t) first * (H / 128) : nullptr;
            g.acc = reinterpret_cast<float*>(t.state + L.acc_g) + (size_t) first * 128;
            u.acc = reinterpret_cast<float*>(t.state + L.acc_u) + (size_t) first * 128;
            g.in_task_begin = 2 * first * (H / 128);
            u.in_task_begin = (2 * first + m) * (H / 128);
            g.out_task_begin = first * (I / 128);
            u.out_task_begin = first * (I / 128);
            g.out = reinterpret_cast<uint32_t*>(t.scratch + L.xd_d) + (size_t) first * I;
            g.out_stride = I;
            g.out_suh = reinterpret_cast<const __half*>(t.du[e]);
            g.out_sblk = t.mul1 ? reinterpret_cast<float*>(t.scratch + L.sb_d) + (size_t) first * (I / 128) : nullptr;
            gu[2 * q] = g;
            gu[2 * q + 1] = u;

            GvProblem d = {};
            d.k = I;
            d.n = H;
            d.m = m;
            d.trellis = reinterpret_cast<const uint32_t*>(t.dt[e]);
            d.suh = nullptr;  // input written already rotated by the SwiGLU epilogue
            d.svh = reinterpret_cast<const __half*>(t.dv[e]);
            d.xd = reinterpret_cast<uint32_t*>(t.scratch + L.xd_d) + (size_t) first * I;
            d.sblk = g.out_sblk;
            d.acc = reinterpret_cast<float*>(t.state + L.acc_d) + (size_t) first * 128;
            d.acc_nb_stride = pmax * 128;
            d.out = t.out;
            d.out_stride = t.out_stride;
            d.out_rows = token + first;
            d.out_scale = weight + first;
            d.out_task_begin = first * (H / 128);
            dn[q] = d;
        }
    }

    if (tid == 0) {
        int* tot = reinterpret_cast<int*>(t.scratch + L.tot);
        // [0..3] gate+up interleaved, [4..7] gate only / up only view, [8..11] swiglu, [12..15] down
        tot[0] = 2 * total_probs; tot[1] = 0; tot[2] = 2 * total_rows * (H / 128); tot[3] = 0;
        tot[4] = total_probs;     tot[5] = 0; tot[6] = 0;                          tot[7] = 0;
        tot[8] = total_probs;     tot[9] = 0; tot[10] = 0; tot[11] = total_rows * (I / 128);
        tot[12] = total_probs;    tot[13] = 0; tot[14] = 0; tot[15] = total_rows * (H / 128);
    }
}

static int launch_route(const MoeTables& t, const MoeLayout& L, cudaStream_t stream)
{
    // the combine epilogue adds into out: zero it over the whole GPU first (a 2D memset,
    // not the single routing CTA)
    if (!t.accumulate &&
        cudaMemset2DAsync(t.out, (size_t) t.out_stride * sizeof(float), 0, (size_t) t.hidden * sizeof(float),
                          (size_t) t.tokens, stream) != cudaSuccess)
        return kErrLaunch;
    exl3_moe_route_kernel<<<1, kRouteThreads, 0, stream>>>(t, L);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrLaunch;
}

// Batched experts (reference p2b_gemv_batched): problem e = expert ids[e] on
// x (shared) or x[e]; table built on the device from the id list.
struct BatchedTables {
    const __half* x;
    long long x_stride;
    int x_per_expert;
    const long long *tp, *sp, *vp;
    int table_size;
    const int* ids;
    int count, m, k, n;
    void* out;
    int out_elem;  // bytes per output element
    GvProblem* tab;
    uint32_t* xd;
    float* sblk;
    float* acc;
};

__global__ void exl3_batched_build_kernel(const BatchedTables b)
{
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= b.count) return;
    int id = b.ids[e];
    id = id < 0 ? 0 : (id >= b.table_size ? b.table_size - 1 : id);  // callers pass clamped ids
    GvProblem p = {};
    p.trellis = reinterpret_cast<const uint32_t*>(b.tp[id]);
    p.suh = reinterpret_cast<const __half*>(b.sp[id]);
    p.svh = reinterpret_cast<const __half*>(b.vp[id]);
    p.x = b.x + (b.x_per_expert ? (size_t) e * b.m * b.x_stride : 0);
    p.x_stride = b.x_stride;
    p.xd = b.xd + (size_t) e * b.m * b.k;
    p.sblk = b.sblk ? b.sblk + (size_t) e * b.m * (b.k / 128) : nullptr;
    p.acc = b.acc + (size_t) e * b.m * 128;
    p.acc_nb_stride = b.count * b.m * 128;
    p.out = reinterpret_cast<char*>(b.out) + (size_t) e * b.m * b.n * b.out_elem;  // [count][m][n]
    p.out_stride = b.n;
    p.k = b.k;
    p.n = b.n;
    p.m = b.m;
    p.in_task_begin = e * b.m * (b.k / 128);
    p.out_task_begin = e * b.m * (b.n / 128);
    b.tab[e] = p;
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" size_t exl3b200_moe_state_size(int max_tokens, int topk, int hidden, int inter)
{
    if (max_tokens < 1 || topk < 1 || hidden % 128 || inter % 128 || max_tokens * topk > kMaxPairs) return 0;
    return moe_layout(max_tokens * topk, hidden, inter).state_bytes;
}

extern "C" size_t exl3b200_moe_scratch_size(int max_tokens, int topk, int hidden, int inter)
{
    if (max_tokens < 1 || topk < 1 || hidden % 128 || inter % 128 || max_tokens * topk > kMaxPairs) return 0;
    return moe_layout(max_tokens * topk, hidden, inter).scratch_bytes;
}

extern "C" int exl3b200_moe(const void* x, long long x_stride, int tokens, int hidden, int inter,
                            const int* topk_ids, const float* topk_weights, int topk, int num_experts,
                            const long long* gate_trellis, const long long* gate_suh, const long long* gate_svh,
                            const long long* up_trellis, const long long* up_suh, const long long* up_svh,
                            const long long* down_trellis, const long long* down_suh, const long long* down_svh,
                            int K_gate, int K_up, int K_down, int cb, float swiglu_limit, float* out,
                            long long out_stride, int accumulate, int max_tokens, void* state, size_t state_bytes,
                            void* scratch, size_t scratch_bytes, void* stream)
{
    if (!x || !topk_ids || !topk_weights || !out || !state || !scratch) return kErrNullPointer;
    if (!gate_trellis || !gate_suh || !gate_svh || !up_trellis || !up_suh || !up_svh || !down_trellis ||
        !down_suh || !down_svh)
        return kErrNullPointer;
    if (tokens < 1 || tokens > max_tokens || topk < 1 || max_tokens * topk > kMaxPairs) return kErrBadShape;
    if (num_experts < 1 || num_experts > kMaxLocalExperts) return kErrBadShape;
    if (hidden <= 0 || inter <= 0 || hidden % 128 || inter % 128 || x_stride < hidden || out_stride < hidden)
        return kErrBadShape;
    for (int Kx : {K_gate, K_up, K_down})
        if (Kx < 2 || Kx > 4) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (((uintptr_t) state & 255) || ((uintptr_t) scratch & 255) || ((uintptr_t) x & 3) || (x_stride & 1))
        return kErrUnaligned;
    const int pmax = max_tokens * topk;
    const MoeLayout L = moe_layout(pmax, hidden, inter);
    if (state_bytes < L.state_bytes || scratch_bytes < L.scratch_bytes) return kErrWorkspace;

    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char* sc = reinterpret_cast<char*>(scratch);
    MoeTables t;
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
    t.state = reinterpret_cast<char*>(state);
    t.tokens = tokens;
    t.topk = topk;
    t.experts = num_experts;
    t.hidden = hidden;
    t.inter = inter;
    t.pmax = pmax;
    t.mul1 = cb == 2;
    t.accumulate = accumulate;
    // few rows per expert (at most 4 on average): problems of up to 8 rows on the
    // one-row-group kernel (8 tiles per warp), whose tile rate is the higher; an expert
    // with more rows then streams its codes once per 8 rows
    t.prob_rows = (long long) tokens * topk <= 4ll * num_experts ? 8 : kGvMaxRows;
    int rc = launch_route(t, L, st);
    if (rc != kOk) return rc;

    const int* tot = reinterpret_cast<const int*>(sc + L.tot);
    const GvProblem* gu = reinterpret_cast<const GvProblem*>(sc + L.tab_gu);
    const GvProblem* dn = reinterpret_cast<const GvProblem*>(sc + L.tab_d);
    const int rows = std::min(tokens, t.prob_rows);
    const int pairs = tokens * topk;

    GvArgs a = {};
    a.dev = gu;
    a.dev_totals = tot;  // [2p, -, in, -]
    a.stride = 1;
    a.offset = 0;
    rc = gv_launch_input(a, 2 * pairs * (hidden / 128), true, st);
    if (rc != kOk) return rc;

    a.uniform_units = (inter / 128) * (hidden / 16);
    if (K_gate == K_up) {
        rc = gv_launch_matmul(a, K_gate, cb, rows, 0, true, st);
    } else {
        a.dev_totals = tot + 4;  // [p, ...]: gate-only / up-only views of the interleaved table
        a.stride = 2;
        a.offset = 0;
        rc = gv_launch_matmul(a, K_gate, cb, rows, 0, true, st);
        if (rc == kOk) {
            a.offset = 1;
            rc = gv_launch_matmul(a, K_up, cb, rows, 0, true, st);
        }
    }
    if (rc != kOk) return rc;

    GvArgs e = {};
    e.dev = gu;
    e.dev_totals = tot + 8;  // swiglu view: gate entries
    e.stride = 2;
    e.offset = 0;
    e.epi_mode = kEpiSwiglu;
    e.swiglu_limit = swiglu_limit;
    rc = gv_launch_epilogue(e, cb, pairs * (inter / 128), true, st);
    if (rc != kOk) return rc;

    GvArgs d = {};
    d.dev = dn;
    d.dev_totals = tot + 12;
    d.stride = 1;
    d.offset = 0;
    d.uniform_units = (hidden / 128) * (inter / 16);
    rc = gv_launch_matmul(d, K_down, cb, rows, 0, true, st);
    if (rc != kOk) return rc;
    d.epi_mode = kEpiCombine;
    return gv_launch_epilogue(d, cb, pairs * (hidden / 128), true, st);
}

extern "C" size_t exl3b200_batched_state_size(int count, int m, int n)
{
    if (count < 1 || m < 1 || m > EXL3B200_GEMV_MAX_M || n % 128) return 0;
    return al256((size_t) (n / 128) * count * m * 128 * sizeof(float));
}

extern "C" size_t exl3b200_batched_scratch_size(int count, int m, int k)
{
    if (count < 1 || m < 1 || m > EXL3B200_GEMV_MAX_M || k % 128) return 0;
    return al256((size_t) count * sizeof(GvProblem)) + al256((size_t) count * m * k * sizeof(uint32_t)) +
           al256((size_t) count * m * (k / 128) * sizeof(float));
}

extern "C" int exl3b200_batched_gemv(const void* x, int x_per_expert, long long x_stride, int m, int k, int n, int K,
                                     int cb, const long long* trellis_ptrs, const long long* suh_ptrs,
                                     const long long* svh_ptrs, int table_size, const int* expert_ids, int count,
                                     void* out, int out_dtype, void* state, size_t state_bytes, void* scratch,
                                     size_t scratch_bytes, void* stream)
{
    if (!x || !trellis_ptrs || !suh_ptrs || !svh_ptrs || !expert_ids || !out || !state || !scratch)
        return kErrNullPointer;
    if (count < 1 || table_size < 1 || m < 1 || m > EXL3B200_GEMV_MAX_M) return kErrBadShape;
    if (k <= 0 || n <= 0 || k % 128 || n % 128 || x_stride < k) return kErrBadShape;
    if (K < 2 || K > 4) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (out_dtype < 0 || out_dtype > 2) return kErrBadArgument;
    if (((uintptr_t) state & 255) || ((uintptr_t) scratch & 255) || ((uintptr_t) x & 3) || (x_stride & 1))
        return kErrUnaligned;
    if (state_bytes < exl3b200_batched_state_size(count, m, n) ||
        scratch_bytes < exl3b200_batched_scratch_size(count, m, k))
        return kErrWorkspace;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char* sc = reinterpret_cast<char*>(scratch);
    BatchedTables b;
    b.x = reinterpret_cast<const __half*>(x);
    b.x_stride = x_stride;
    b.x_per_expert = x_per_expert;
    b.tp = trellis_ptrs;
    b.sp = suh_ptrs;
    b.vp = svh_ptrs;
    b.table_size = table_size;
    b.ids = expert_ids;
    b.count = count;
    b.m = m;
    b.k = k;
    b.n = n;
    b.out = out;
    b.out_elem = out_dtype == 2 ? 4 : 2;
    b.tab = reinterpret_cast<GvProblem*>(sc);
    sc += al256((size_t) count * sizeof(GvProblem));
    b.xd = reinterpret_cast<uint32_t*>(sc);
    sc += al256((size_t) count * m * k * sizeof(uint32_t));
    b.sblk = cb == 2 ? reinterpret_cast<float*>(sc) : nullptr;
    b.acc = reinterpret_cast<float*>(state);
    exl3_batched_build_kernel<<<(count + 127) / 128, 128, 0, st>>>(b);
    if (cudaGetLastError() != cudaSuccess) return kErrLaunch;

    GvArgs a = {};
    a.dev = b.tab;
    a.nprob = count;
    a.in_tasks = count * m * (k / 128);
    a.out_tasks = count * m * (n / 128);
    a.stride = 1;
    a.uniform_units = (n / 128) * (k / 16);
    a.out_dtype = out_dtype;
    a.epi_mode = kEpiStore;
    int rc = gv_launch_input(a, a.in_tasks, true, st);
    if (rc != kOk) return rc;
    rc = gv_launch_matmul(a, K, cb, m, 0, true, st);
    if (rc != kOk) return rc;
    return gv_launch_epilogue(a, cb, a.out_tasks, true, st);
}
