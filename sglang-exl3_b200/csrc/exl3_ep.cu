// Expert-parallel routed MoE with the dispatch and the combine done by this
// library's own kernels over NVLink peer memory (no NCCL, no host synchronisation).
//
// The reference leaves expert parallelism to SGLang's dispatcher around its MoE
// method (src/sglang_exl3/exl3.py:2254-2313, expert ids mapped to local ones by
// exl3.py:485-509).  Here W ranks each own E / W experts (rank r: global experts
// [r E/W, (r+1) E/W)) and each holds its own T tokens.  One call, stream-ordered:
//
//   plan      (1 CTA)  which ranks own an expert of each token; the row index of the
//                      token in every such rank's receive region for this rank
//   dispatch  (grid)   each token row goes ONCE to every rank owning one of its
//                      experts (peer stores of the fp16 row, its k ids rewritten to
//                      that rank's local ids or -1, its k weights); then a system
//                      fence and one arrival per CTA on every rank's counter
//   receive   (grid)   bounded wait for every rank's arrivals; ids of the unused rows
//                      of every region set to -1
//   MoE                the local routed SwiGLU pipeline (small-M or tensor-core, by
//                      the shape map) over the W receive regions as one row list
//   return    (grid)   every result row (fp32, already weighted) pushed back into
//                      the source rank's return region; fence; arrivals
//   combine   (grid)   bounded wait; out[t] = sum over the ranks t went to of their
//                      result rows, in rank order
//
// Shared buffer of every rank (allocated once, mapped into every rank by IPC):
//   [control 128 B][counters 128 B: dispatch and return arrivals, two parities]
//   then per parity: counts [W] int32, ids [W][T][k] int32, weights [W][T][k] fp32,
//   rows [W][T][H] fp16 (region s: rows sent by rank s), returns [W][T][H] fp32
//   (region d: results computed by rank d).
// Calls alternate between the two parities.  A rank reaches call c + 2 only after
// every rank returned its call c + 1 results, which needs every rank's call c + 1
// dispatch, so no rank still reads parity c data when it is overwritten.  Waits are
// bounded (exl3b200_set_wait_limit; default 2 s); a wait that runs out records
// EXL3B200_ETIMEOUT in the device status and poisons the buffer (later calls skip
// the exchange and return zeros) until exl3b200_peer_reset.
#include <algorithm>

#include "exl3_common.cuh"
#include "exl3_capi_internal.h"
#include "exl3_epilogue.cuh"

namespace exl3b200 {

constexpr int kEpMaxRanks = 8;
constexpr int kEpGrid = 128;     // CTAs of the exchange kernels (the same on every rank)
constexpr int kEpThreads = 256;
constexpr unsigned long long kEpTimeoutNs = 2000000000ull;

struct EpCtl {
    unsigned int epoch;     // calls completed
    unsigned int done_rx;   // CTAs of the running receive that finished
    unsigned int done_cb;   // CTAs of the running combine that finished
    unsigned int poisoned;
};

struct EpLayout {
    size_t counts, ids, w, rows, ret, parity, total;
};

static EpLayout ep_layout(int world, int max_tokens, int topk, int hidden)
{
    auto al = [](size_t v) { return (v + 255) & ~(size_t) 255; };
    EpLayout L;
    const size_t W = world, T = max_tokens, k = topk, H = hidden;
    size_t o = 0;
    L.counts = o; o += al(W * 4);
    L.ids = o; o += al(W * T * k * 4);
    L.w = o; o += al(W * T * k * 4);
    L.rows = o; o += al(W * T * H * 2);
    L.ret = o; o += al(W * T * H * 4);
    L.parity = o;
    L.total = 256 + 2 * o;
    return L;
}

struct EpArgsDev {
    char* buf[kEpMaxRanks];  // every rank's buffer as mapped here; [rank] = own
    int world, rank, tokens, max_tokens, topk, hidden, per_rank, experts;
    EpLayout L;
    const int* ids;          // [tokens][k] global expert ids
    const float* weights;    // [tokens][k]
    const __half* x;         // [tokens][hidden]
    long long x_stride;
    int* send_idx;           // [tokens][world] row index in each rank's region, -1 when not sent
    int* send_count;         // [world]
    uint4* moe_x;            // [world * max_tokens][hidden / 8] local MoE input rows (fp16)
    int* moe_ids;            // [world * max_tokens][k] local expert ids, -1 for unused rows
    float* moe_w;            // [world * max_tokens][k]
    const float* moe_out;    // [world * max_tokens][hidden] local MoE results
    float* out;              // [tokens][hidden]
    long long out_stride;
    unsigned long long wait_ns;
    int* status;
};

__device__ __forceinline__ EpCtl* ep_ctl(const EpArgsDev& a, int q) { return reinterpret_cast<EpCtl*>(a.buf[q]); }

__device__ __forceinline__ unsigned int* ep_flag(const EpArgsDev& a, int q, int kind, unsigned int parity)
{
    return reinterpret_cast<unsigned int*>(a.buf[q] + 128) + 2 * kind + parity;
}

__device__ __forceinline__ char* ep_area(const EpArgsDev& a, int q, unsigned int parity)
{
    return a.buf[q] + 256 + (size_t) parity * a.L.parity;
}

__device__ __forceinline__ unsigned int ep_parity(const EpArgsDev& a)
{
    return (*reinterpret_cast<volatile unsigned int*>(&ep_ctl(a, a.rank)->epoch) + 1u) & 1u;
}

__device__ __forceinline__ bool ep_poisoned(const EpArgsDev& a)
{
    return *reinterpret_cast<volatile unsigned int*>(&ep_ctl(a, a.rank)->poisoned) != 0u;
}

__device__ __forceinline__ int ep_owner(const EpArgsDev& a, int id)
{
    return (id >= 0 && id < a.experts) ? id / a.per_rank : -1;
}

// Bounded wait of thread 0 until the counter reaches `expect`; false (status and
// poison recorded) when the limit passed first.
__device__ bool ep_wait(const EpArgsDev& a, const unsigned int* cnt, unsigned int expect)
{
    const unsigned long long t0 = globaltimer_ns();
    while (ld_acquire_sys(cnt) < expect) {
        if (globaltimer_ns() - t0 > a.wait_ns) {
            if (a.status) atomicCAS(a.status, 0, (int) kErrTimeout);
            atomicExch(&ep_ctl(a, a.rank)->poisoned, 1u);
            return false;
        }
        __nanosleep(64);
    }
    return true;
}

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------

// Which ranks own an expert of each token, and the token's row in each such rank's
// receive region for this rank (its place among this rank's tokens sent there).
__global__ __launch_bounds__(1024) void exl3_ep_plan_kernel(const __grid_constant__ EpArgsDev a)
{
    __shared__ int s_warp[32][kEpMaxRanks];
    __shared__ int s_base[kEpMaxRanks];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid < kEpMaxRanks) s_base[tid] = 0;
    __syncthreads();
    for (int t0 = 0; t0 < a.tokens; t0 += 1024) {
        const int t = t0 + tid;
        unsigned int mask = 0;
        if (t < a.tokens) {
            for (int j = 0; j < a.topk; ++j) {
                const int d = ep_owner(a, a.ids[(size_t) t * a.topk + j]);
                if (d >= 0) mask |= 1u << d;
            }
        }
        int prefix[kEpMaxRanks];
        for (int d = 0; d < a.world; ++d) {
            const unsigned int b = __ballot_sync(0xffffffffu, (mask >> d) & 1u);
            prefix[d] = __popc(b & ((1u << lane) - 1u));
            if (lane == 0) s_warp[warp][d] = __popc(b);
        }
        __syncthreads();
        if (tid < a.world) {  // exclusive scan of the warp totals, per rank
            int run = s_base[tid];
            for (int w = 0; w < 32; ++w) {
                const int c = s_warp[w][tid];
                s_warp[w][tid] = run;
                run += c;
            }
            s_base[tid] = run;
        }
        __syncthreads();
        if (t < a.tokens)
            for (int d = 0; d < a.world; ++d)
                a.send_idx[(size_t) t * a.world + d] = ((mask >> d) & 1u) ? s_warp[warp][d] + prefix[d] : -1;
        __syncthreads();
    }
    if (tid < a.world) a.send_count[tid] = s_base[tid];
}

// Each (token, rank) row of the plan: the fp16 row, the k ids local to that rank (-1
// for experts elsewhere) and the k weights, stored into the rank's region for this
// rank.  Then the counts, a system fence and one arrival per CTA on every rank.
__global__ __launch_bounds__(kEpThreads) void exl3_ep_dispatch_kernel(const __grid_constant__ EpArgsDev a)
{
    griddep_wait();
    if (ep_poisoned(a)) return;
    const unsigned int par = ep_parity(a);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kEpThreads / 32);
    const int H = a.hidden, k = a.topk;
    for (int task = blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5); task < a.tokens * a.world; task += warps) {
        const int t = task / a.world, d = task - t * a.world;
        const int i = a.send_idx[(size_t) t * a.world + d];
        if (i < 0) continue;
        char* area = ep_area(a, d, par);
        const size_t row = (size_t) a.rank * a.max_tokens + i;
        const uint4* src = reinterpret_cast<const uint4*>(a.x + (size_t) t * a.x_stride);
        uint4* dst = reinterpret_cast<uint4*>(area + a.L.rows) + row * (H / 8);
        for (int c = lane; c < H / 8; c += 32) dst[c] = src[c];
        if (lane < k) {
            const int id = a.ids[(size_t) t * k + lane];
            const bool mine = ep_owner(a, id) == d;
            reinterpret_cast<int*>(area + a.L.ids)[row * k + lane] = mine ? id - d * a.per_rank : -1;
            reinterpret_cast<float*>(area + a.L.w)[row * k + lane] = a.weights[(size_t) t * k + lane];
        }
    }
    if (blockIdx.x == 0 && threadIdx.x < a.world)
        reinterpret_cast<int*>(ep_area(a, threadIdx.x, par) + a.L.counts)[a.rank] = a.send_count[threadIdx.x];
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < a.world)
        asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(ep_flag(a, threadIdx.x, 0, par)) : "memory");
}

// Every rank's rows are in: they are copied from this call's parity area into the
// fixed local input of the MoE pipeline (so the pipeline's launches do not depend on
// the parity, and a CUDA graph of a call replays for either), with ids -1 for the
// unused rows of every region (the MoE router skips them).  The last CTA re-arms
// the counter.
__global__ __launch_bounds__(kEpThreads) void exl3_ep_receive_kernel(const __grid_constant__ EpArgsDev a)
{
    griddep_wait();
    __shared__ int ok;
    const unsigned int par = ep_parity(a);
    if (threadIdx.x == 0)
        ok = ep_poisoned(a) ? 0 : (ep_wait(a, ep_flag(a, a.rank, 0, par), (unsigned int) (a.world * gridDim.x)) ? 1 : 0);
    __syncthreads();
    const char* area = ep_area(a, a.rank, par);
    const int* counts = reinterpret_cast<const int*>(area + a.L.counts);
    const int* rids = reinterpret_cast<const int*>(area + a.L.ids);
    const float* rw = reinterpret_cast<const float*>(area + a.L.w);
    const uint4* rx = reinterpret_cast<const uint4*>(area + a.L.rows);
    const int lane = threadIdx.x & 31, k = a.topk, H8 = a.hidden / 8;
    const int warps = gridDim.x * (kEpThreads / 32);
    for (int row = blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5); row < a.world * a.max_tokens; row += warps) {
        const int s = row / a.max_tokens, i = row - s * a.max_tokens;
        const bool used = ok && i < __ldcv(counts + s);
        if (lane < k) {
            a.moe_ids[(size_t) row * k + lane] = used ? __ldcv(rids + (size_t) row * k + lane) : -1;
            a.moe_w[(size_t) row * k + lane] = used ? __ldcv(rw + (size_t) row * k + lane) : 0.f;
        }
        if (used)
            for (int c = lane; c < H8; c += 32) a.moe_x[(size_t) row * H8 + c] = __ldcv(rx + (size_t) row * H8 + c);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        EpCtl* ctl = ep_ctl(a, a.rank);
        if (atomicAdd(&ctl->done_rx, 1u) == gridDim.x - 1) {
            ctl->done_rx = 0u;
            if (ok) *ep_flag(a, a.rank, 0, par) = 0u;
        }
    }
}

// Every local result row goes back into its source rank's return region for this
// rank; then the fence and one arrival per CTA on every rank.
__global__ __launch_bounds__(kEpThreads) void exl3_ep_return_kernel(const __grid_constant__ EpArgsDev a)
{
    griddep_wait();
    if (ep_poisoned(a)) return;
    const unsigned int par = ep_parity(a);
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kEpThreads / 32);
    const int H = a.hidden;
    const int* counts = reinterpret_cast<const int*>(ep_area(a, a.rank, par) + a.L.counts);
    for (int task = blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5); task < a.world * a.max_tokens; task += warps) {
        const int s = task / a.max_tokens, i = task - s * a.max_tokens;
        if (i >= __ldcv(counts + s)) continue;
        const float4* src = reinterpret_cast<const float4*>(a.moe_out + (size_t) task * H);
        float4* dst = reinterpret_cast<float4*>(ep_area(a, s, par) + a.L.ret) +
                      ((size_t) a.rank * a.max_tokens + i) * (H / 4);
        for (int c = lane; c < H / 4; c += 32) dst[c] = src[c];
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x < a.world)
        asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(ep_flag(a, threadIdx.x, 1, par)) : "memory");
}

// Every rank's results are in: out[t] = sum, in rank order, of the result rows of the
// ranks t was sent to.  The last CTA re-arms the counter and ends the call (epoch).
__global__ __launch_bounds__(kEpThreads) void exl3_ep_combine_kernel(const __grid_constant__ EpArgsDev a)
{
    griddep_wait();
    __shared__ int ok;
    const unsigned int par = ep_parity(a);
    if (threadIdx.x == 0)
        ok = ep_poisoned(a) ? 0 : (ep_wait(a, ep_flag(a, a.rank, 1, par), (unsigned int) (a.world * gridDim.x)) ? 1 : 0);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kEpThreads / 32);
    const int H = a.hidden;
    const float4* ret = reinterpret_cast<const float4*>(ep_area(a, a.rank, par) + a.L.ret);
    for (int t = blockIdx.x * (kEpThreads / 32) + (threadIdx.x >> 5); t < a.tokens; t += warps) {
        float4* o = reinterpret_cast<float4*>(a.out + (size_t) t * a.out_stride);
        for (int c = lane; c < H / 4; c += 32) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ok) {
                for (int d = 0; d < a.world; ++d) {
                    const int i = a.send_idx[(size_t) t * a.world + d];
                    if (i < 0) continue;
                    const float4 v = __ldcv(ret + ((size_t) d * a.max_tokens + i) * (H / 4) + c);
                    acc.x += v.x;
                    acc.y += v.y;
                    acc.z += v.z;
                    acc.w += v.w;
                }
            }
            o[c] = acc;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        EpCtl* ctl = ep_ctl(a, a.rank);
        if (atomicAdd(&ctl->done_cb, 1u) == gridDim.x - 1) {
            ctl->done_cb = 0u;
            if (ok) {
                *ep_flag(a, a.rank, 1, par) = 0u;
                __threadfence();
                volatile unsigned int* ep = reinterpret_cast<volatile unsigned int*>(&ctl->epoch);
                *ep = *ep + 1u;
            }
        }
    }
}

}  // namespace exl3b200

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
using namespace exl3b200;

namespace {

struct EpScratch {
    size_t send_idx, send_count, moe_x, moe_ids, moe_w, moe_out, moe, total;
};

size_t al256(size_t v) { return (v + 255) & ~(size_t) 255; }

int ep_path(const exl3b200_ep_args& p, int world)
{
    if (p.path == 0 || p.path == 1) return p.path;
    const int local = p.experts / world;
    return exl3b200_select_shape(p.tokens, p.hidden, p.inter, p.K_gate, p.cb, local, p.topk) == EXL3B200_SHAPE_MOE_TC
               ? 1
               : 0;
}

int ep_sizes(const exl3b200_ep_args& p, int world, int path, EpScratch* sc, size_t* state)
{
    const int rows = world * p.max_tokens;
    const int local = p.experts / world;
    size_t moe_scratch, moe_state = 0;
    if (path == 1) {
        moe_scratch = exl3b200_moe_tc_scratch_size(rows, p.topk, local, p.hidden, p.inter);
    } else {
        moe_scratch = exl3b200_moe_scratch_size(rows, p.topk, p.hidden, p.inter);
        moe_state = exl3b200_moe_state_size(rows, p.topk, p.hidden, p.inter);
    }
    if (moe_scratch == 0 || (path == 0 && moe_state == 0)) return kErrBadShape;
    size_t o = 0;
    sc->send_idx = o; o += al256((size_t) p.max_tokens * world * 4);
    sc->send_count = o; o += al256((size_t) world * 4);
    sc->moe_x = o; o += al256((size_t) rows * p.hidden * 2);
    sc->moe_ids = o; o += al256((size_t) rows * p.topk * 4);
    sc->moe_w = o; o += al256((size_t) rows * p.topk * 4);
    sc->moe_out = o; o += al256((size_t) rows * p.hidden * 4);
    sc->moe = o; o += al256(moe_scratch);
    sc->total = o;
    *state = moe_state;
    return kOk;
}

int ep_check(const exl3b200_ep_args* p, const exl3b200_peers* peers)
{
    if (!p || !peers) return kErrNullPointer;
    if (peers->world < 1 || peers->world > kEpMaxRanks || peers->rank < 0 || peers->rank >= peers->world)
        return kErrBadArgument;
    if (p->experts < peers->world || p->experts % peers->world) return kErrBadShape;
    if (p->tokens < 0 || p->tokens > p->max_tokens || p->max_tokens < 1) return kErrBadShape;
    if (p->topk < 1 || p->topk > 32 || p->hidden % 128 || p->inter % 128 || p->hidden <= 0 || p->inter <= 0)
        return kErrBadShape;
    if (peers->max_rows != p->max_tokens || peers->hidden != p->hidden) return kErrBadShape;
    return kOk;
}

}  // namespace

extern "C" size_t exl3b200_ep_buffer_size(int world, int max_tokens, int topk, int hidden)
{
    if (world < 1 || world > kEpMaxRanks || max_tokens < 1 || topk < 1 || topk > 32 || hidden <= 0 || hidden % 128)
        return 0;
    return ep_layout(world, max_tokens, topk, hidden).total;
}

extern "C" int exl3b200_ep_workspace(const exl3b200_ep_args* p, const exl3b200_peers* peers, size_t* state_bytes,
                                     size_t* scratch_bytes)
{
    int rc = ep_check(p, peers);
    if (rc != kOk) return rc;
    if (!state_bytes || !scratch_bytes) return kErrNullPointer;
    EpScratch sc;
    rc = ep_sizes(*p, peers->world, ep_path(*p, peers->world), &sc, state_bytes);
    *scratch_bytes = sc.total;
    return rc;
}

extern "C" int exl3b200_ep_moe(const exl3b200_ep_args* p, const exl3b200_peers* peers, void* state,
                               size_t state_bytes, void* scratch, size_t scratch_bytes, void* stream)
{
    int rc = ep_check(p, peers);
    if (rc != kOk) return rc;
    if (!p->x || !p->topk_ids || !p->topk_weights || !p->out || !scratch || !p->tables) return kErrNullPointer;
    for (int i = 0; i < 9; ++i)
        if (!p->tables[i]) return kErrNullPointer;
    for (int q = 0; q < peers->world; ++q) {
        if (!peers->buffers[q]) return kErrNullPointer;
        if ((uintptr_t) peers->buffers[q] & 255) return kErrUnaligned;
    }
    if (((uintptr_t) p->x & 15) || (p->x_stride % 8) || ((uintptr_t) p->out & 15) || (p->out_stride % 4))
        return kErrUnaligned;
    if (((uintptr_t) scratch & 255) || ((uintptr_t) state & 255)) return kErrUnaligned;
    const int W = peers->world;
    const int path = ep_path(*p, W);
    EpScratch sc;
    size_t need_state = 0;
    rc = ep_sizes(*p, W, path, &sc, &need_state);
    if (rc != kOk) return rc;
    if (scratch_bytes < sc.total || state_bytes < need_state || (need_state && !state)) return kErrWorkspace;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    char* sp = reinterpret_cast<char*>(scratch);

    EpArgsDev a = {};
    for (int q = 0; q < W; ++q) a.buf[q] = reinterpret_cast<char*>(peers->buffers[q]);
    a.world = W;
    a.rank = peers->rank;
    a.tokens = p->tokens;
    a.max_tokens = p->max_tokens;
    a.topk = p->topk;
    a.hidden = p->hidden;
    a.experts = p->experts;
    a.per_rank = p->experts / W;
    a.L = ep_layout(W, p->max_tokens, p->topk, p->hidden);
    a.ids = p->topk_ids;
    a.weights = p->topk_weights;
    a.x = reinterpret_cast<const __half*>(p->x);
    a.x_stride = p->x_stride;
    a.send_idx = reinterpret_cast<int*>(sp + sc.send_idx);
    a.send_count = reinterpret_cast<int*>(sp + sc.send_count);
    a.moe_x = reinterpret_cast<uint4*>(sp + sc.moe_x);
    a.moe_ids = reinterpret_cast<int*>(sp + sc.moe_ids);
    a.moe_w = reinterpret_cast<float*>(sp + sc.moe_w);
    a.moe_out = reinterpret_cast<const float*>(sp + sc.moe_out);
    a.out = p->out;
    a.out_stride = p->out_stride;
    a.wait_ns = wait_limit_ns(kEpTimeoutNs);
    a.status = exl3_status_dev_ptr();
    if (!a.status) return kErrLaunch;

    exl3_ep_plan_kernel<<<1, 1024, 0, st>>>(a);
    exl3_ep_dispatch_kernel<<<kEpGrid, kEpThreads, 0, st>>>(a);
    exl3_ep_receive_kernel<<<kEpGrid, kEpThreads, 0, st>>>(a);
    if (cudaPeekAtLastError() != cudaSuccess) return kErrLaunch;

    // the local experts over the W regions as one list of W * max_tokens rows (the
    // unused ones carry ids -1); one row per (source rank, token), weights applied
    const int rows = W * p->max_tokens;
    const long long* const* tb = reinterpret_cast<const long long* const*>(p->tables);
    float* moe_out = reinterpret_cast<float*>(sp + sc.moe_out);
    if (path == 1) {
        rc = exl3b200_moe_tc(sp + sc.moe_x, p->hidden, rows, p->hidden, p->inter, a.moe_ids, a.moe_w, p->topk,
                             a.per_rank, tb[0], tb[1], tb[2], tb[3], tb[4], tb[5], tb[6], tb[7], tb[8], p->K_gate,
                             p->K_up, p->K_down, p->cb, p->swiglu_limit, moe_out, p->hidden, 0, rows, sp + sc.moe,
                             scratch_bytes - sc.moe, stream);
    } else {
        rc = exl3b200_moe(sp + sc.moe_x, p->hidden, rows, p->hidden, p->inter, a.moe_ids, a.moe_w, p->topk,
                          a.per_rank, tb[0], tb[1], tb[2], tb[3], tb[4], tb[5], tb[6], tb[7], tb[8], p->K_gate,
                          p->K_up, p->K_down, p->cb, p->swiglu_limit, moe_out, p->hidden, 0, rows, state,
                          state_bytes, sp + sc.moe, scratch_bytes - sc.moe, stream);
    }
    if (rc != kOk) return rc;

    exl3_ep_return_kernel<<<kEpGrid, kEpThreads, 0, st>>>(a);
    exl3_ep_combine_kernel<<<kEpGrid, kEpThreads, 0, st>>>(a);
    return cudaPeekAtLastError() == cudaSuccess ? kOk : kErrLaunch;
}
