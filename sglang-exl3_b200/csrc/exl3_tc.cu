// Large-M EXL3 matmul on the 5th-generation tensor cores (tcgen05 MMA with TMEM
// accumulators): y = H128(H128(x * suh) @ W_raw) * svh / 128 for m rows at once.
//
// Replaces the reference's exl3_gemm for M > 8 (csrc/exl3_gemm.cu:9-31, which
// runs the upstream exllamav3 smem-decode GEMM) and the dense part of its fat
// GEMM (csrc/exl3_fat_gemm.cu:65-305).  Three kernels, chained by programmatic
// dependent launch:
//
// * exl3_tc_input_kernel: one warp per (row, 128-block) computes the fp16
//   x_had = H128(x * suh) / sqrt(128) with the reference's roundings (the same
//   rotate_block as the small-M path) and writes it straight into the shared
//   memory image the MMA reads: 128-row x 64-column blocks of 16 KB, rows of 128
//   bytes whose 16-byte chunks are XOR-swizzled by (row % 8) (the canonical
//   K-major SWIZZLE_128B layout).  Padding rows up to a multiple of 128 are zero.
// * exl3_tc_gemm_kernel: persistent, one CTA per SM, stream-K: the output is cut
//   into 256x256 tiles (rows fastest, so CTAs working on one column block's codes
//   run together and share them in L2), every tile into k/64 iterations, and the
//   concatenated iteration list into one contiguous range per CTA.  A CTA's range
//   is a sequence of segments (a tile's iterations [kc0, kc1)).  Warp roles
//   (warp w runs on SM sub-partition w % 4):
//     warp 0    allocates 512 TMEM columns; lane 0 streams the activation blocks
//               with bulk copies (cp.async.bulk) into a 3-stage ring;
//     warp 1    lane 0 issues tcgen05.mma (M=128, N=256, K=16, fp16 x fp16 -> fp32)
//               for each of the two 128-row accumulators and releases ring slots
//               with tcgen05.commit;
//     warp 2    lane 0 streams the trellis codes of the tile (4 k-tiles x 16
//               n-tiles per stage) with bulk copies into a 4-stage ring;
//     warps 3-23 with w % 4 != 1 (16 warps) decode the codes from shared memory
//               (window extraction, codebook, final fp16 add / fma; one 16-column
//               tile x 4 k-tiles per warp and stage) into the B operand (256
//               output columns x 64 k, K-major, 128-byte swizzle, 3-stage ring);
//     warps 5, 9, .., 21 share the MMA issuer's sub-partition and only run the
//               epilogue of TMEM lanes 32..63: a decoder there took issue slots
//               from the MMA issuer (measured: MMA issue time halved without it).
//   At the end of a segment each thread of the epilogue owns one TMEM lane
//   (= output row); H128 over a 128-column block is a 32-point transform per
//   quarter in registers, written back to TMEM, then the stride-32 and stride-64
//   butterflies on 8-column slices; scale by svh / sqrt(128).  A segment that is a
//   whole tile stores the output; a part of a tile split between CTAs adds its
//   fp32 partial into the tile's slot of a zeroed state buffer (the transform is
//   linear).
// * exl3_tc_finish_kernel: converts the split tiles' slots to the output dtype
//   and re-zeroes them.
// * exl3_tc_pair_kernel: the same matmul on 2-CTA clusters (tcgen05.mma.cta_group::2,
//   512 x 256 tiles) for large M, where each decoded code tile then feeds 512 rows.
// Every wait on an mbarrier is bounded (1 s of %globaltimer); a wait that runs
// out raises the CTA's abort flag and the library's sticky device status; every
// role then leaves its loop, waits (bounded) for its own copies and MMAs in
// flight, and the CTA frees its TMEM and exits.
//
// The same kernel runs grouped launches (template MODE 1 and 2, used by the
// routed-MoE pipeline and the routed combine in exl3_tc_moe.cu): many problems
// with shared k, n, K and codebook, whose tile list, problem table and tile
// count an earlier kernel wrote to device memory.  Every role looks up the
// problem of a segment's tile; activation rows come from the problem's
// k-chunk-major image, one bulk copy of its (8-rounded) rows per 128-row
// accumulator and 64-k chunk; the epilogue stores fp32 rows (MODE 1; split tiles
// add into zeroed rows) or adds weight * y into out[token] (MODE 2).  No slots
// and no finish kernel.
#include <algorithm>

#include "exl3_common.cuh"
#include "exl3_capi_internal.h"
#include "exl3_tc_internal.h"

namespace exl3b200 {

// Warp roles (warp w runs on SM sub-partition w % 4): 0 activation producer,
// 1 MMA issuer, 2 code producer; of warps 3..23, those with w % 4 == 1 share the
// MMA issuer's sub-partition and only run the epilogue of TMEM lanes 32..63 (so
// no decoder competes with the MMA issuer for issue slots); the other 16 decode.
constexpr int kTcWarps = 24;
constexpr int kTcDecWarps = 16;
constexpr int kTcThreads = 32 * kTcWarps;  // 768
constexpr int kTcRows = 256;          // rows per tile: two M=128 accumulators
constexpr int kTcCols = 256;          // output columns per tile
constexpr int kTcStageA = 3;
constexpr int kTcStageB = 3;
constexpr int kTcStageT = 4;
constexpr int kTcABlock = 128 * 64 * 2;        // one 128-row x 64-k fp16 block (16 KB)
constexpr int kTcBStage = kTcCols * 64 * 2;    // 32 KB
constexpr int kTcSlotFloats = kTcRows * kTcCols;  // one split tile's fp32 partial sums
constexpr unsigned long long kTcTimeoutNs = 1000000000ull;

__device__ int g_exl3_device_status = 0;  // sticky: first device-side error code

template <int K>
struct TcSmem {
    static constexpr int kBars = 2 * kTcStageA + 2 * kTcStageT + 2 * kTcStageB + 4;
    static constexpr uint32_t kTChunk = 4u * 16u * 32u * K;  // codes of one stage at 256 columns
    static constexpr uint32_t kA = 0;
    static constexpr uint32_t kB = kA + kTcStageA * 2 * kTcABlock;
    static constexpr uint32_t kT = kB + kTcStageB * kTcBStage;
    static constexpr uint32_t kBar = kT + kTcStageT * kTChunk;
    static constexpr uint32_t kMisc = kBar + 8 * kBars;
    static constexpr uint32_t kBytes = kMisc + 16;
    static constexpr uint32_t kLaunchBytes = kBytes + 1024;  // room to align the base to 1024
};

struct TcArgs {
    const uint8_t* xt;        // swizzled rotated input blocks [m128 tiles][k/64][16 KB]
    const uint8_t* trellis;   // [k/16][n/16][32K bytes]
    const __half* svh;        // [n], 16-byte aligned
    void* out;
    float* slots;             // zeroed [grid][256][256] fp32: partial sums of split tiles
    long long out_stride;     // elements
    long long iters;          // tiles * k/64
    int m, k, n;
    int mtiles, tiles, nkc;
    int out_dtype;            // 0 fp16, 1 bf16, 2 fp32
    int vec_store;            // rows of out are 16-byte aligned
    int pair;                 // exl3_tc_pair_kernel launch: 512-row tiles, slots per CTA of each pair
    // grouped launches (kTcGroupedStore / kTcGroupedCombine): the problem of each
    // tile and the tile count come from device memory written by an earlier kernel
    const TcProblem* probs;
    const int* tile_prob;
    const int* dev_tiles;
    const int* dev_tile_base;  // nullable
    long long xt_rows;         // rows of the k-chunk-major input image
    const int* slot_token;     // combine: output row of each routed slot
    const float* slot_weight;  // combine: its routing weight
    unsigned long long wait_ns;  // limit of every bounded barrier wait
    // kTcDenseSwiglu: n = 2 * inter (gate columns, then up columns of the trellis);
    // tiles pair gate block j with up block j; the epilogue writes the down projection's
    // input image (the exl3_tc_input_kernel layout, k = inter)
    uint8_t* img;              // down input image [mpad/128][inter/64][16 KB]
    const __half* suh2;        // down projection suh [inter]
    float swiglu_limit;        // 0 or infinite: no clip
    int inter;
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tc_griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void tc_griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t) __cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_n(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Slow path of a bounded wait: false once the CTA's abort flag is up
// (check_abort) or the deadline passes (then raises the flag and the status).  The
// CTA's wait limit sits in shared memory 4 bytes after its abort flag.
__device__ __forceinline__ bool mbar_test_sleep(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 200000;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag, bool check_abort)
{
    const unsigned long long t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_test_sleep(bar, parity)) return true;
        if ((it & 63u) == 0) {
            if (check_abort && *abort_flag) return false;
            if (global_ns() - t0 > *reinterpret_cast<volatile unsigned long long*>(
                                       reinterpret_cast<volatile char*>(abort_flag) + 4)) {
                *abort_flag = 1;
                atomicCAS(&g_exl3_device_status, 0, (int) kErrTimeout);
                return false;
            }
        }
    }
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, bool check_abort)
{
    if (mbar_test(bar, parity)) return true;
    return mbar_wait_slow(bar, parity, abort_flag, check_abort);
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t slot, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// --- CTA pairs (cta_group::2): one MMA spans the TMEM and shared memory of both CTAs of
// a 2-CTA cluster.  A rows are split between the CTAs (M / 2 each, same shared memory
// offset), B columns likewise (N / 2 each); the leader (cluster rank 0) issues.
__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address in the shared::cluster window of the variable at `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

// Arrive on an mbarrier of another CTA of the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// try_wait with acquire at cluster scope (for barriers that another CTA arrives on).
__device__ __forceinline__ bool mbar_test_cl(uint32_t bar, uint32_t parity, uint32_t hint_ns)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

__device__ __noinline__ bool mbar_wait_cl_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag)
{
    const unsigned long long t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_test_cl(bar, parity, 200000u)) return true;
        if ((it & 63u) == 0) {
            if (*abort_flag) return false;
            if (global_ns() - t0 > *reinterpret_cast<volatile unsigned long long*>(
                                       reinterpret_cast<volatile char*>(abort_flag) + 4)) {
                *abort_flag = 1;
                atomicCAS(&g_exl3_device_status, 0, (int) kErrTimeout);
                return false;
            }
        }
    }
}

__device__ __forceinline__ bool mbar_wait_cl(uint32_t bar, uint32_t parity, volatile int* abort_flag)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    return mbar_wait_cl_slow(bar, parity, abort_flag);
}

__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Completion of the pair MMAs issued so far arrives on the mbarrier at this offset in
// both CTAs of the pair.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar)
{
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"((uint16_t) 3)
        : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16 inputs, fp32 accumulate)
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8])
{
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float (&v)[8])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
                 "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                 "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4])
{
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const float (&v)[4])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
                 "r"(__float_as_uint(v[3]))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024
// bytes apart (SBO), leading offset unused for swizzled K-major (1), version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr)
{
    const uint32_t lo = ((saddr >> 4) & 0x3FFFu) | (1u << 16);
    const uint32_t hi = (1024u >> 4) | (1u << 14) | (2u << 29);
    return ((uint64_t) hi << 32) | lo;
}

// Instruction descriptor, kind::f16: fp32 D, fp16 A and B, both K-major, M = 128
// (M = 256 for a CTA pair).
__device__ __forceinline__ uint32_t tc_idesc(int n, int m = 128)
{
    return (1u << 4) | ((uint32_t) (n >> 3) << 17) | ((uint32_t) (m >> 4) << 24);
}

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b)
{
    uint32_t r;
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c)
{
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// The 8 fp16 weights of a lane in one tile, packed as the k pairs (j, j+1):
// h2[0] = (k0, k0+1) at n0, h2[1] = (k0+8, k0+9) at n0, h2[2], h2[3] the same at
// n0 + 8, with k0 = 2 (lane % 4), n0 = lane / 4.  Round to nearest, exactly as
// codebook_value_rn (one fp16 rounding of an exact sum / fma).
template <int K, int CB>
__device__ __forceinline__ void tc_decode_lane(uint32_t wa, uint32_t wb, int shift7, uint32_t (&h2)[4])
{
    uint32_t w[8];
    lane_windows<K>(wa, wb, shift7, w);
    uint32_t p[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) p[j] = codebook_pre<CB>(w[j]);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t lo = prmt(p[2 * q], p[2 * q + 1], 0x5410);
        if constexpr (CB == 2) {
            h2[q] = hfma2_u32(lo, (uint32_t) kMul1InvBits * 0x10001u, (uint32_t) kMul1BiasBits * 0x10001u);
        } else {
            const uint32_t hi = prmt(p[2 * q], p[2 * q + 1], 0x7632);
            h2[q] = hadd2_u32(lo, hi);
        }
    }
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr)
{
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ void sts_u32(uint32_t addr, uint32_t v)
{
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// One warp's share of a stage: NB16 = 16 n-tiles (256 columns): n-tile dw, k-tiles
// 0..3; NB16 = 8 (128 columns): n-tile dw % 8, k-tiles 2 (dw / 8) + {0, 1}.  tch and
// bst are shared-memory addresses of the stage's codes and B operand (explicit
// shared-space loads and stores).
template <int K, int CB, int NB16>
__device__ __forceinline__ void tc_decode_stage(uint32_t tch, uint32_t bst, int dw, int lane, const LaneWords& lw)
{
    constexpr int T = NB16 / 4;
    const int ntl = NB16 == 16 ? dw : (dw & 7);
    const int kt0 = NB16 == 16 ? 0 : 2 * (dw >> 3);
    const uint32_t tw = tch + (uint32_t) ((kt0 * NB16 + ntl) * 32 * K);
    uint32_t wa[T], wb[T];
#pragma unroll
    for (int i = 0; i < T; ++i) {
        wa[i] = lds_u32(tw + 4u * (uint32_t) (i * NB16 * 8 * K + lw.wa));
        wb[i] = lds_u32(tw + 4u * (uint32_t) (i * NB16 * 8 * K + lw.wb));
    }
    const int sw = lane >> 2;
    const uint32_t rowp = bst + (uint32_t) (ntl * 16 * 128 + (lane >> 2) * 128 + 4 * (lane & 3));
#pragma unroll
    for (int i = 0; i < T; ++i) {
        uint32_t h2[4];
        tc_decode_lane<K, CB>(wa[i], wb[i], lw.shift7, h2);
        const int kt = kt0 + i;
        const uint32_t c_lo = (uint32_t) (((2 * kt) ^ sw) << 4), c_hi = (uint32_t) (((2 * kt + 1) ^ sw) << 4);
        sts_u32(rowp + c_lo, h2[0]);
        sts_u32(rowp + c_hi, h2[1]);
        sts_u32(rowp + 1024 + c_lo, h2[2]);
        sts_u32(rowp + 1024 + c_hi, h2[3]);
    }
}

// ---------------------------------------------------------------------------
// input stage
// ---------------------------------------------------------------------------
__global__ __launch_bounds__(256) void exl3_tc_input_kernel(const __half* __restrict__ x, long long x_stride,
                                                            const __half* __restrict__ suh, int m, int mpad, int k,
                                                            uint8_t* __restrict__ xt)
{
    tc_griddep_launch();
    tc_griddep_wait();
    const int lane = threadIdx.x & 31;
    const int nblk = k >> 7;
    const int nkc = k >> 6;
    const int tasks = mpad * nblk;
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int task = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); task < tasks; task += warps) {
        const int r = task / nblk;
        const int b = task - r * nblk;
        __half h[4];
        if (r < m) {
            rotate_block(x + (size_t) r * x_stride + b * 128, suh ? suh + b * 128 : nullptr, lane, h);
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) h[i] = __ushort_as_half(0);
        }
        const int rr = r & 127;
        uint8_t* tile_row = xt + ((size_t) (r >> 7) * nkc << 14) + rr * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int kc = 2 * b + (i >> 1);
            const int kk = lane + 32 * (i & 1);
            *reinterpret_cast<__half*>(tile_row + ((size_t) kc << 14) + (((kk >> 3) ^ (rr & 7)) << 4) + (kk & 7) * 2) =
                h[i];
        }
    }
}

// ---------------------------------------------------------------------------
// epilogue
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fwht32_local(float (&v)[32])
{
#pragma unroll
    for (int s = 1; s < 32; s <<= 1) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if ((i & s) == 0) {
                const float a = v[i], b = v[i + s];
                v[i] = __fadd_rn(a, b);
                v[i + s] = __fsub_rn(a, b);
            }
        }
    }
}

__device__ __forceinline__ void store8(const TcArgs& a, int row, int col, const float (&v)[8])
{
    if (a.out_dtype == 2) {
        float* dst = reinterpret_cast<float*>(a.out) + (size_t) row * a.out_stride + col;
        if (a.vec_store) {
            reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) dst[i] = v[i];
        }
        return;
    }
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if (a.out_dtype == 0) {
            const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
            pk[i] = *reinterpret_cast<const uint32_t*>(&h);
        } else {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            pk[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
    }
    uint16_t* dst = reinterpret_cast<uint16_t*>(a.out) + (size_t) row * a.out_stride + col;
    if (a.vec_store) {
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            dst[2 * i] = (uint16_t) (pk[i] & 0xffffu);
            dst[2 * i + 1] = (uint16_t) (pk[i] >> 16);
        }
    }
}

// One 128-column block of one 128-row accumulator, this warp's 32 rows.  TMEM
// lanes = rows; the block's columns are overwritten (the transform runs in place).
__device__ __forceinline__ void tc_epilogue_block(const TcArgs& a, uint32_t taddr, int row, int col0, bool whole,
                                                  float* __restrict__ slot_row)
{
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
        float v[32];
        tmem_ld32(taddr + 32 * j, v);
        tmem_ld_wait();
        fwht32_local(v);
        tmem_st32(taddr + 32 * j, v);
    }
    tmem_st_wait();
    const uint4* sv4 = reinterpret_cast<const uint4*>(a.svh + col0);
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
        float u[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j) tmem_ld8(taddr + 32 * j + 8 * c, u[j]);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float b0 = __fadd_rn(u[0][i], u[1][i]), b1 = __fsub_rn(u[0][i], u[1][i]);
            const float b2 = __fadd_rn(u[2][i], u[3][i]), b3 = __fsub_rn(u[2][i], u[3][i]);
            u[0][i] = __fadd_rn(b0, b2);
            u[2][i] = __fsub_rn(b0, b2);
            u[1][i] = __fadd_rn(b1, b3);
            u[3][i] = __fsub_rn(b1, b3);
        }
        if (row >= a.m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 s = __ldg(sv4 + 4 * j + c);
            const __half* sh = reinterpret_cast<const __half*>(&s);
#pragma unroll
            for (int i = 0; i < 8; ++i) u[j][i] = u[j][i] * kHadScale * __half2float(sh[i]);
            const int col = 32 * j + 8 * c;
            if (whole) {
                store8(a, row, col0 + col, u[j]);
            } else {
                float4* dst = reinterpret_cast<float4*>(slot_row + col);
                atomicAdd(dst, make_float4(u[j][0], u[j][1], u[j][2], u[j][3]));
                atomicAdd(dst + 1, make_float4(u[j][4], u[j][5], u[j][6], u[j][7]));
            }
        }
    }
}

// Grouped launches: one 128-column block of one 128-row accumulator, this warp's
// 32 rows, the same transform as tc_epilogue_block; then dst (row < m; null
// otherwise) receives w * y, stored when PLAIN (a whole tile of a store launch),
// else added with vector atomics.
template <bool PLAIN>
__device__ __forceinline__ void tc_epilogue_block_grouped(uint32_t taddr, const __half* __restrict__ svh,
                                                          float* __restrict__ dst, float w)
{
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
        float v[32];
        tmem_ld32(taddr + 32 * j, v);
        tmem_ld_wait();
        fwht32_local(v);
        tmem_st32(taddr + 32 * j, v);
    }
    tmem_st_wait();
    const uint4* sv4 = reinterpret_cast<const uint4*>(svh);
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
        float u[4][8];
#pragma unroll
        for (int j = 0; j < 4; ++j) tmem_ld8(taddr + 32 * j + 8 * c, u[j]);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float b0 = __fadd_rn(u[0][i], u[1][i]), b1 = __fsub_rn(u[0][i], u[1][i]);
            const float b2 = __fadd_rn(u[2][i], u[3][i]), b3 = __fsub_rn(u[2][i], u[3][i]);
            u[0][i] = __fadd_rn(b0, b2);
            u[2][i] = __fsub_rn(b0, b2);
            u[1][i] = __fadd_rn(b1, b3);
            u[3][i] = __fsub_rn(b1, b3);
        }
        if (!dst) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 s = __ldg(sv4 + 4 * j + c);
            const __half* sh = reinterpret_cast<const __half*>(&s);
#pragma unroll
            for (int i = 0; i < 8; ++i) u[j][i] = w * (u[j][i] * kHadScale * __half2float(sh[i]));
            float4* d4 = reinterpret_cast<float4*>(dst + 32 * j + 8 * c);
            const float4 lo = make_float4(u[j][0], u[j][1], u[j][2], u[j][3]);
            const float4 hi = make_float4(u[j][4], u[j][5], u[j][6], u[j][7]);
            if constexpr (PLAIN) {
                d4[0] = lo;
                d4[1] = hi;
            } else {
                atomicAdd(d4, lo);
                atomicAdd(d4 + 1, hi);
            }
        }
    }
}

// In-place 128-point transform of one TMEM block (this thread's row): 32-point
// transforms of the four 32-column quarters; the stride-32 and stride-64 butterflies
// run where the block is read back (tc_block_final).
__device__ __forceinline__ void tc_block_fwht32(uint32_t taddr)
{
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
        float v[32];
        tmem_ld32(taddr + 32 * j, v);
        tmem_ld_wait();
        fwht32_local(v);
        tmem_st32(taddr + 32 * j, v);
    }
}

// Columns 32 j + 8 c + i (j < 4, i < 8) of a block after tc_block_fwht32: the last
// two butterfly stages, unscaled.
__device__ __forceinline__ void tc_block_final(uint32_t taddr, int c, float (&u)[4][8])
{
#pragma unroll
    for (int j = 0; j < 4; ++j) tmem_ld8(taddr + 32 * j + 8 * c, u[j]);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float b0 = __fadd_rn(u[0][i], u[1][i]), b1 = __fsub_rn(u[0][i], u[1][i]);
        const float b2 = __fadd_rn(u[2][i], u[3][i]), b3 = __fsub_rn(u[2][i], u[3][i]);
        u[0][i] = __fadd_rn(b0, b2);
        u[2][i] = __fsub_rn(b0, b2);
        u[1][i] = __fadd_rn(b1, b3);
        u[3][i] = __fsub_rn(b1, b3);
    }
}

// The same for the 4 columns 32 j + 4 c + i (c < 8, i < 4).
__device__ __forceinline__ void tc_block_final4(uint32_t taddr, int c, float (&u)[4][4])
{
#pragma unroll
    for (int j = 0; j < 4; ++j) tmem_ld4(taddr + 32 * j + 4 * c, u[j]);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float b0 = __fadd_rn(u[0][i], u[1][i]), b1 = __fsub_rn(u[0][i], u[1][i]);
        const float b2 = __fadd_rn(u[2][i], u[3][i]), b3 = __fsub_rn(u[2][i], u[3][i]);
        u[0][i] = __fadd_rn(b0, b2);
        u[2][i] = __fsub_rn(b0, b2);
        u[1][i] = __fadd_rn(b1, b3);
        u[3][i] = __fsub_rn(b1, b3);
    }
}

// Clipped SwiGLU of one element, rounded to fp16 where the reference keeps the
// activation (csrc/p2b_moe.cu:304-313; src/sglang_exl3/exl3.py:1207-1215), then the
// down projection's fp16 pre-scale x * suh (its input transform's first rounding).
__device__ __forceinline__ float swiglu_pre(float g, float u, float lim, float suh)
{
    if (lim > 0.f && lim < 3.0e38f) {
        g = fminf(g, lim);
        u = fminf(fmaxf(u, -lim), lim);
    }
    const float act = __half2float(__float2half_rn(g / (1.0f + expf(-g)) * u));
    return __half2float(__float2half_rn(__fmul_rn(act, suh)));
}

// 8 consecutive columns of the down projection's input, / sqrt(128) and rounded to
// fp16 (the last rounding of exl3_tc_input_kernel), packed as one 16-byte chunk of an
// input image row.
__device__ __forceinline__ uint4 tc_pack8(const float (&v)[8])
{
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h = __floats2half2_rn(__fmul_rn(v[2 * i], kHadScale), __fmul_rn(v[2 * i + 1], kHadScale));
        pk[i] = *reinterpret_cast<const uint32_t*>(&h);
    }
    return make_uint4(pk[0], pk[1], pk[2], pk[3]);
}

// Named barrier of the two epilogue warps of one accumulator in one TMEM lane quarter
// (ids 1..8; id 0 is __syncthreads), with the tcgen05 fences that order their TMEM
// accesses around it.
__device__ __forceinline__ void tc_pair_sync(int id)
{
    tc_fence_before();
    asm volatile("bar.sync %0, 64;" ::"r"(id) : "memory");
    tc_fence_after();
}

// 32-point transforms of quarters j0, j0 + 1 of one TMEM block (this thread's row).
__device__ __forceinline__ void tc_block_fwht32_half(uint32_t taddr, int j0)
{
#pragma unroll 1
    for (int j = j0; j < j0 + 2; ++j) {
        float v[32];
        tmem_ld32(taddr + 32 * j, v);
        tmem_ld_wait();
        fwht32_local(v);
        tmem_st32(taddr + 32 * j, v);
    }
}

// SwiGLU epilogue of one 128-row accumulator of a gate|up tile (kTcDenseSwiglu,
// kTcGroupedSwiglu), shared by two warps of the same TMEM lane quarter (role 0 and 1;
// 32 rows): TMEM columns 0..127 hold the gate block j, 128..255 the up block j.
// Whole tiles: y = H128(acc) * svh / sqrt(128) for both blocks, the clipped SwiGLU
// rounded to fp16, x * suh of the down projection rounded to fp16, written back over
// the gate block, then its 128-point transform, / sqrt(128) and one fp16 rounding; the
// caller's store(col, chunk) puts each 8-column chunk into the down projection's input
// image (the roundings of exl3_tc_input_kernel).  Split tiles add y of both blocks
// into the slot row; the finish kernel completes them.  Each phase is halved between
// the two warps (role 0 transforms the gate block, role 1 the up block, then each
// takes half of the column slices).
template <class Store>
__device__ __forceinline__ void tc_epilogue_swiglu(uint32_t taddr, int role, int bar_id, const __half* svh_gate,
                                                   const __half* svh_up, const __half* suh_down, float lim,
                                                   bool whole, float* __restrict__ slot_row, bool row_ok,
                                                   Store store)
{
    tc_block_fwht32(taddr + 128 * role);
    tmem_st_wait();
    tc_pair_sync(bar_id);
    const uint2* svg = reinterpret_cast<const uint2*>(svh_gate);
    const uint2* svu = reinterpret_cast<const uint2*>(svh_up);
    const uint2* su2 = reinterpret_cast<const uint2*>(suh_down);
    // 4-column slices keep the gate and up values of a slice within the register budget
#pragma unroll 1
    for (int c = 4 * role; c < 4 * role + 4; ++c) {
        float g[4][4], u[4][4];
        tc_block_final4(taddr, c, g);
        tc_block_final4(taddr + 128, c, u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint2 sg4 = __ldg(svg + 8 * j + c), su4 = __ldg(svu + 8 * j + c);
            const __half* sg = reinterpret_cast<const __half*>(&sg4);
            const __half* sup = reinterpret_cast<const __half*>(&su4);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                g[j][i] = g[j][i] * kHadScale * __half2float(sg[i]);
                u[j][i] = u[j][i] * kHadScale * __half2float(sup[i]);
            }
            if (whole) {
                const uint2 s24 = __ldg(su2 + 8 * j + c);
                const __half* s2 = reinterpret_cast<const __half*>(&s24);
#pragma unroll
                for (int i = 0; i < 4; ++i) g[j][i] = swiglu_pre(g[j][i], u[j][i], lim, __half2float(s2[i]));
                tmem_st4(taddr + 32 * j + 4 * c, g[j]);
            } else if (row_ok) {
                const int col = 32 * j + 4 * c;
                atomicAdd(reinterpret_cast<float4*>(slot_row + col), make_float4(g[j][0], g[j][1], g[j][2], g[j][3]));
                atomicAdd(reinterpret_cast<float4*>(slot_row + 128 + col),
                          make_float4(u[j][0], u[j][1], u[j][2], u[j][3]));
            }
        }
    }
    if (!whole) return;  // uniform over the pair (same segment)
    tmem_st_wait();
    tc_pair_sync(bar_id);
    tc_block_fwht32_half(taddr, 2 * role);
    tmem_st_wait();
    tc_pair_sync(bar_id);
#pragma unroll 1
    for (int c = 2 * role; c < 2 * role + 2; ++c) {
        float p[4][8];
        tc_block_final(taddr, c, p);
#pragma unroll
        for (int j = 0; j < 4; ++j) store(32 * j + 8 * c, tc_pack8(p[j]));
    }
}

// What a CTA needs to know about the tile of a segment: the dense launch's single
// problem, or the grouped launch's problem of that tile.
struct TcSeg {
    const uint8_t* xt;  // grouped: the problem's input image
    const uint8_t* trellis;
    const __half* svh;
    float* gout;  // grouped store: fp32 output of the problem's row 0
    int m, mt, nt, row0, slot0;
    // kTcGroupedSwiglu: the up projection's image, codes and svh; the down projection's suh
    const uint8_t* xt2;
    const uint8_t* trellis2;
    const __half* svh2;
    const __half* suh2;
};

template <int MODE>
__device__ __forceinline__ TcSeg tc_seg(const TcArgs& a, int tile)
{
    TcSeg s;
    if constexpr (MODE == kTcDense || MODE == kTcDenseSwiglu) {
        s.xt = a.xt;
        s.trellis = a.trellis;
        s.svh = a.svh;
        s.gout = nullptr;
        s.m = a.m;
        s.mt = tile % a.mtiles;
        s.nt = tile / a.mtiles;
        s.row0 = 0;
        s.slot0 = 0;
    } else {
        const TcProblem& p = a.probs[a.tile_prob[tile]];
        const int local = tile - p.tile_begin;
        s.xt = p.xt;
        s.trellis = p.trellis;
        s.svh = p.svh;
        s.gout = p.out;
        s.m = p.m;
        s.mt = local % p.mtiles;
        s.nt = local / p.mtiles;
        s.row0 = p.row0;
        s.slot0 = p.slot0;
        if constexpr (MODE == kTcGroupedSwiglu) {
            const TcProblem& u = a.probs[a.tile_prob[tile] + 1];
            s.xt2 = u.xt;
            s.trellis2 = u.trellis;
            s.svh2 = u.svh;
            s.suh2 = p.suh2;
        }
    }
    return s;
}

// Work of CTA c: two contiguous ranges of the iteration list (tile-major, k-chunk
// minor).  First whole tiles, w = tiles / grid per CTA, so the CTAs of this phase
// all start at k = 0 and walk k together: the activation and code chunks that the
// concurrent tiles share are read from DRAM about once and then hit in L2 (with
// every CTA at a different k, as in a plain stream-K split, the working set is the
// whole input image plus all codes, which does not fit in L2 at large m).  Then the
// remaining tiles' iterations are split evenly over the grid (stream-K); only
// these tiles can be split between CTAs.
struct TcRanges {
    long long b[2], e[2];
    long long sk0;  // first iteration of the stream-K phase
};

// Whole tiles only (an epilogue that cannot be split): contiguous runs of tiles,
// balanced to within one tile.
__device__ __forceinline__ TcRanges tc_ranges_whole(long long iters, int nkc, int grid, int c)
{
    TcRanges r;
    const long long tiles = iters / nkc;
    r.b[0] = tiles * c / grid * nkc;
    r.e[0] = tiles * (c + 1) / grid * nkc;
    r.b[1] = r.e[1] = r.sk0 = iters;
    return r;
}

__device__ __forceinline__ TcRanges tc_ranges(long long iters, int nkc, int grid, int c)
{
    TcRanges r;
    const long long w = iters / nkc / grid;
    r.sk0 = w * grid * nkc;
    r.b[0] = (long long) c * w * nkc;
    r.e[0] = r.b[0] + w * nkc;
    const long long rem = iters - r.sk0;
    r.b[1] = r.sk0 + rem * c / grid;
    r.e[1] = r.sk0 + rem * (c + 1) / grid;
    return r;
}

// the CTA whose stream-K range holds iteration it (it >= sk0): its slot collects
// the partial sums of the tile that starts there
__device__ __forceinline__ int tc_cta_of(long long iters, int nkc, int grid, long long it)
{
    const long long sk0 = iters / nkc / grid * grid * nkc;
    return (int) (((it - sk0 + 1) * grid - 1) / (iters - sk0));
}

// ---------------------------------------------------------------------------
// matmul
// ---------------------------------------------------------------------------
template <int K, int CB, int MODE>
__global__ __launch_bounds__(kTcThreads, 1) void exl3_tc_gemm_kernel(const __grid_constant__ TcArgs a)
{
    constexpr int SA = kTcStageA, ST = kTcStageT;  // activation and code ring depths
    using L = TcSmem<K>;
    static_assert(L::kLaunchBytes <= 232448, "shared memory per CTA");
    extern __shared__ uint8_t tc_smem_raw[];
    const uint32_t raw = smem_u32(tc_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = tc_smem_raw + (base - raw);
    const uint32_t sA = base + L::kA, sB = base + L::kB, sT = base + L::kT, sBar = base + L::kBar;
    const uint32_t full_a = sBar, empty_a = full_a + 8 * SA;
    const uint32_t full_t = empty_a + 8 * SA, empty_t = full_t + 8 * ST;
    const uint32_t full_b = empty_t + 8 * ST, empty_b = full_b + 8 * kTcStageB;
    // accumulator barriers: full / empty of TMEM buffer 0 (columns 0..255, or all 512 for
    // two 128-row accumulators), then of buffer 1 (columns 256..511; kTcGroupedSwiglu
    // alternates the buffers by segment, so a tile's epilogue overlaps the next tile's MMAs)
    const uint32_t acc_full = empty_b + 8 * kTcStageB, acc_empty = acc_full + 8;
    constexpr bool kDblAcc = MODE == kTcGroupedSwiglu;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + L::kMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + L::kMisc + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int grid = gridDim.x;
    const int nkc = a.nkc;

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            mbar_init(full_a + 8 * s, 1);
            mbar_init(empty_a + 8 * s, 1);
        }
        for (int s = 0; s < ST; ++s) {
            mbar_init(full_t + 8 * s, 1);
            mbar_init(empty_t + 8 * s, kTcDecWarps);
        }
        for (int s = 0; s < kTcStageB; ++s) {
            mbar_init(full_b + 8 * s, kTcDecWarps);
            mbar_init(empty_b + 8 * s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + 16 * b, 1);
            // every decoder and epilogue-only warp; kTcGroupedSwiglu: 6 (see the arrival)
            mbar_init(acc_empty + 16 * b, kDblAcc ? 6 : kTcWarps - 3);
        }
        *abort_flag = 0;
        *reinterpret_cast<volatile unsigned long long*>(gbase + L::kMisc + 8) = a.wait_ns;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        tmem_alloc(base + L::kMisc, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    tc_griddep_launch();
    long long iters = a.iters;
    int tile_base = 0;
    constexpr bool kGrouped = MODE == kTcGroupedStore || MODE == kTcGroupedCombine || MODE == kTcGroupedSwiglu;
    constexpr bool kSwiglu = MODE == kTcDenseSwiglu || MODE == kTcGroupedSwiglu;
    if constexpr (kGrouped) {
        tc_griddep_wait();  // the routing kernel wrote the tile list, the problems and the counts
        iters = (long long) *reinterpret_cast<const volatile int*>(a.dev_tiles) * nkc;
        if (a.dev_tile_base) tile_base = *reinterpret_cast<const volatile int*>(a.dev_tile_base);
    }
    const TcRanges rg = MODE == kTcGroupedSwiglu ? tc_ranges_whole(iters, nkc, grid, blockIdx.x)
                                                 : tc_ranges(iters, nkc, grid, blockIdx.x);

    if (warp == 0) {
        // activation producer
        tc_griddep_wait();  // the input stage of this call wrote xt
        if (lane == 0) {
            uint32_t s = 0, ph = 0, used = 0, par = 0;  // ring slot, phase; per-slot issued / parity bits
            bool ok = true;
            for (int r = 0; r < 2; ++r)
            for (long long it = rg.b[r], it_end = rg.e[r]; it < it_end && ok;) {
                const int tile = (int) (it / nkc), kc0 = (int) (it - (long long) tile * nkc);
                const int kc1 = (int) min((long long) nkc, kc0 + (it_end - it));
                const TcSeg sg = tc_seg<MODE>(a, tile + tile_base);
                const int mt = sg.mt;
                const int rows_t = min(kTcRows, sg.m - mt * kTcRows);
                const int nacc = rows_t > 128 ? 2 : 1;
                if constexpr (MODE == kTcGroupedSwiglu) {
                    // 96-row tiles into rows 32..127 of the A blocks (TMEM lanes 32..127): the gate
                    // image's rows into block 0, the up image's into block 1.  Rows 0..31 keep stale
                    // data; their accumulator rows are never read.
                    const int rows_g = min(kTcSwRows, sg.m - mt * kTcSwRows);
                    const uint32_t b0 = (uint32_t) ((rows_g + 7) & ~7) * 128u;
                    const size_t row = (size_t) sg.row0 + (size_t) mt * kTcSwRows;
                    for (int kc = kc0; kc < kc1; ++kc) {
                        if (!mbar_wait(empty_a + 8 * s, ph ^ 1, abort_flag, true)) { ok = false; break; }
                        const size_t off = ((size_t) kc * (size_t) a.xt_rows + row) * 128;
                        mbar_expect_tx(full_a + 8 * s, 2 * b0);
                        bulk_g2s(sA + (s * 2) * kTcABlock + 32 * 128, sg.xt + off, b0, full_a + 8 * s);
                        bulk_g2s(sA + (s * 2 + 1) * kTcABlock + 32 * 128, sg.xt2 + off, b0, full_a + 8 * s);
                        used |= 1u << s;
                        par = (par & ~(1u << s)) | (ph << s);
                        if (++s == SA) { s = 0; ph ^= 1; }
                    }
                } else if constexpr (MODE == kTcDense || MODE == kTcDenseSwiglu) {
                    const uint8_t* src0 = a.xt + (((size_t) (2 * mt) * nkc + kc0) << 14);
                    const size_t acc_step = (size_t) nkc << 14;
                    for (int kc = kc0; kc < kc1; ++kc, src0 += kTcABlock) {
                        if (!mbar_wait(empty_a + 8 * s, ph ^ 1, abort_flag, true)) { ok = false; break; }
                        mbar_expect_tx(full_a + 8 * s, (uint32_t) (nacc * kTcABlock));
                        bulk_g2s(sA + (s * 2) * kTcABlock, src0, kTcABlock, full_a + 8 * s);
                        if (nacc == 2) bulk_g2s(sA + (s * 2 + 1) * kTcABlock, src0 + acc_step, kTcABlock, full_a + 8 * s);
                        used |= 1u << s;
                        par = (par & ~(1u << s)) | (ph << s);
                        if (++s == SA) { s = 0; ph ^= 1; }
                    }
                } else {
                    // only the problem's rows (rounded up to 8) of each 128-row block; the
                    // accumulator rows past them hold garbage that no epilogue stores
                    const uint32_t b0 = (uint32_t) ((min(128, rows_t) + 7) & ~7) * 128u;
                    const uint32_t b1 = rows_t > 128 ? (uint32_t) ((rows_t - 128 + 7) & ~7) * 128u : 0u;
                    const size_t row = (size_t) sg.row0 + (size_t) mt * kTcRows;
                    for (int kc = kc0; kc < kc1; ++kc) {
                        if (!mbar_wait(empty_a + 8 * s, ph ^ 1, abort_flag, true)) { ok = false; break; }
                        const uint8_t* src = sg.xt + ((size_t) kc * (size_t) a.xt_rows + row) * 128;
                        mbar_expect_tx(full_a + 8 * s, b0 + b1);
                        bulk_g2s(sA + (s * 2) * kTcABlock, src, b0, full_a + 8 * s);
                        if (b1) bulk_g2s(sA + (s * 2 + 1) * kTcABlock, src + 128 * 128, b1, full_a + 8 * s);
                        used |= 1u << s;
                        par = (par & ~(1u << s)) | (ph << s);
                        if (++s == SA) { s = 0; ph ^= 1; }
                    }
                }
                it += kc1 - kc0;
            }
            // own copies in flight (all consumed already unless the CTA aborted)
            for (uint32_t j = 0; j < SA; ++j)
                if (used >> j & 1) mbar_wait(full_a + 8 * j, par >> j & 1, abort_flag, false);
        }
    } else if (warp == 2) {
        // code producer
        if (lane == 0) {
            const size_t row_bytes = (size_t) (a.n >> 4) * 32 * K;
            uint32_t s = 0, ph = 0, used = 0, par = 0;
            bool ok = true;
            for (int r = 0; r < 2; ++r)
            for (long long it = rg.b[r], it_end = rg.e[r]; it < it_end && ok;) {
                const int tile = (int) (it / nkc), kc0 = (int) (it - (long long) tile * nkc);
                const int kc1 = (int) min((long long) nkc, kc0 + (it_end - it));
                const TcSeg sg = tc_seg<MODE>(a, tile + tile_base);
                const int nt = sg.nt;
                const int bn = kSwiglu ? kTcCols : min(kTcCols, a.n - nt * kTcCols);
                const uint32_t seg = (uint32_t) (bn >> 4) * 32 * K;
                // swiglu: gate tiles 8 nt .. 8 nt + 7, then the same up tiles (dense: inter / 16
                // tiles further on in the fused trellis; grouped: in the up problem's trellis)
                const size_t col_off = kSwiglu ? (size_t) nt * 8 * 32 * K : (size_t) nt * 16 * 32 * K;
                const uint8_t* src = sg.trellis + (size_t) kc0 * 4 * row_bytes + col_off;
                const uint8_t* src_up = MODE == kTcGroupedSwiglu
                                            ? sg.trellis2 + (size_t) kc0 * 4 * row_bytes + col_off
                                            : src + (size_t) (a.inter >> 4) * 32 * K;
                for (int kc = kc0; kc < kc1; ++kc, src += 4 * row_bytes, src_up += 4 * row_bytes) {
                    if (!mbar_wait(empty_t + 8 * s, ph ^ 1, abort_flag, true)) { ok = false; break; }
                    mbar_expect_tx(full_t + 8 * s, 4 * seg);
                    const uint32_t dst = sT + s * L::kTChunk;
                    if constexpr (kSwiglu) {
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            bulk_g2s(dst + i * seg, src + i * row_bytes, seg / 2, full_t + 8 * s);
                            bulk_g2s(dst + i * seg + seg / 2, src_up + i * row_bytes, seg / 2, full_t + 8 * s);
                        }
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; ++i) bulk_g2s(dst + i * seg, src + i * row_bytes, seg, full_t + 8 * s);
                    }
                    used |= 1u << s;
                    par = (par & ~(1u << s)) | (ph << s);
                    if (++s == ST) { s = 0; ph ^= 1; }
                }
                it += kc1 - kc0;
            }
            for (uint32_t j = 0; j < ST; ++j)
                if (used >> j & 1) mbar_wait(full_t + 8 * j, par >> j & 1, abort_flag, false);
        }
    } else if (warp == 1) {
        // MMA issuer
        if (lane == 0) {
            uint32_t sa = 0, pa = 0, sb = 0, pb = 0;
            int seg_i = 0;
            bool ok = true;
            const uint64_t a_desc0 = sw128_desc(sA), b_desc0 = sw128_desc(sB);
            for (int r = 0; r < 2; ++r)
            for (long long it = rg.b[r], it_end = rg.e[r]; it < it_end && ok; ++seg_i) {
                const int tile = (int) (it / nkc), kc0 = (int) (it - (long long) tile * nkc);
                const int kc1 = (int) min((long long) nkc, kc0 + (it_end - it));
                const TcSeg sg = tc_seg<MODE>(a, tile + tile_base);
                const int mt = sg.mt, nt = sg.nt;
                const int nacc = MODE == kTcGroupedSwiglu ? 1 : (sg.m - mt * kTcRows > 128 ? 2 : 1);
                const uint32_t idesc = tc_idesc(MODE == kTcGroupedSwiglu ? 128
                                                : MODE == kTcDenseSwiglu ? kTcCols
                                                                         : min(kTcCols, a.n - nt * kTcCols));
                // the epilogue of the previous segment has read the accumulators
                const int buf = kDblAcc ? (seg_i & 1) : 0;
                const uint32_t use = (uint32_t) (kDblAcc ? seg_i >> 1 : seg_i);
                const uint32_t tacc = tmem + (uint32_t) (256 * buf);
                if (!mbar_wait(acc_empty + 16 * buf, (use & 1) ^ 1, abort_flag, true)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kc = kc0; kc < kc1; ++kc) {
                    if (!mbar_wait(full_a + 8 * sa, pa, abort_flag, true) ||
                        !mbar_wait(full_b + 8 * sb, pb, abort_flag, true)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    // descriptor start addresses advance in 16-byte units: 32 bytes per k-step
                    const uint64_t ad = a_desc0 + sa * (2 * kTcABlock >> 4);
                    const uint64_t bd = b_desc0 + sb * (kTcBStage >> 4);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint32_t acc_flag = (kc != kc0 || ks != 0) ? 1u : 0u;
                        if constexpr (MODE == kTcGroupedSwiglu) {
                            // gate columns 0..127 from A block 0, up columns 128..255 (B rows
                            // 128.., 16 KB on) from A block 1
                            tc_mma(tacc, ad + 2 * ks, bd + 2 * ks, idesc, acc_flag);
                            tc_mma(tacc + 128, ad + (kTcABlock >> 4) + 2 * ks, bd + (16384 >> 4) + 2 * ks, idesc,
                                   acc_flag);
                        } else {
                            tc_mma(tmem, ad + 2 * ks, bd + 2 * ks, idesc, acc_flag);
                            if (nacc == 2)
                                tc_mma(tmem + 256, ad + (kTcABlock >> 4) + 2 * ks, bd + 2 * ks, idesc, acc_flag);
                        }
                    }
                    tc_commit(empty_a + 8 * sa);
                    tc_commit(empty_b + 8 * sb);
                    if (++sa == SA) { sa = 0; pa ^= 1; }
                    if (++sb == kTcStageB) { sb = 0; pb ^= 1; }
                }
                tc_commit(acc_full + 16 * buf);
                it += kc1 - kc0;
            }
            // every MMA issued by this thread has completed before the CTA frees TMEM
            // (a commit tracks all of the thread's earlier tcgen05 operations)
            if (seg_i > 0) {
                const int last = seg_i - 1;
                const int buf = kDblAcc ? (last & 1) : 0;
                const uint32_t use = (uint32_t) (kDblAcc ? last >> 1 : last);
                mbar_wait(acc_full + 16 * buf, use & 1, abort_flag, false);
            }
        }
    } else {
        // decoders (and the epilogue of their TMEM lane quarter) or epilogue-only
        // warps of lane quarter 1
        const int q = warp & 3;                               // TMEM lane quarter this warp may access
        const int hq = q == 3 ? warp >> 2 : (warp >> 2) - 1;  // its index among the quarter's warps
        const bool decoder = q != 1;
        const int dw = (warp - 3) - (warp - 2) / 4;           // decoder index 0..15

        tc_griddep_wait();
        const LaneWords lw = lane_words<K>(lane);
        uint32_t st = 0, pt = 0, sb = 0, pb = 0;
        int seg_i = 0;
        bool ok = true;
        for (int r = 0; r < 2; ++r)
        for (long long it = rg.b[r], it_end = rg.e[r]; it < it_end && ok; ++seg_i) {
            const int tile = (int) (it / nkc), kc0 = (int) (it - (long long) tile * nkc);
            const int kc1 = (int) min((long long) nkc, kc0 + (it_end - it));
            const TcSeg sg = tc_seg<MODE>(a, tile + tile_base);
            const int mt = sg.mt, nt = sg.nt;
            const int bn = kSwiglu ? kTcCols : min(kTcCols, a.n - nt * kTcCols);
            if (decoder) {
                for (int kc = kc0; kc < kc1; ++kc) {
                    if (!mbar_wait(full_t + 8 * st, pt, abort_flag, true) ||
                        !mbar_wait(empty_b + 8 * sb, pb ^ 1, abort_flag, true)) {
                        ok = false;
                        break;
                    }
                    const uint32_t tch = sT + st * L::kTChunk;
                    const uint32_t bst = sB + sb * kTcBStage;
                    if (bn == kTcCols) tc_decode_stage<K, CB, 16>(tch, bst, dw, lane, lw);
                    else tc_decode_stage<K, CB, 8>(tch, bst, dw, lane, lw);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(full_b + 8 * sb);
                        mbar_arrive(empty_t + 8 * st);
                    }
                    if (++st == ST) { st = 0; pt ^= 1; }
                    if (++sb == kTcStageB) { sb = 0; pb ^= 1; }
                }
            }
            const int buf = kDblAcc ? (seg_i & 1) : 0;
            const uint32_t use = (uint32_t) (kDblAcc ? seg_i >> 1 : seg_i);
            const int nacc = MODE == kTcGroupedSwiglu ? 1 : (sg.m - mt * kTcRows > 128 ? 2 : 1);
            const int nblk = bn >> 7;  // swiglu: tasks (accumulator, role) instead of (accumulator, block)
            // kTcGroupedSwiglu: a tile's rows sit in TMEM lanes 32..127 (quarters 1..3); only the
            // two warps of a quarter holding rows wait for the accumulator, the others go on
            // decoding the next tile (the accumulators are double-buffered)
            const bool duty = MODE == kTcGroupedSwiglu
                                  ? (q > 0 && hq < 2 && (q - 1) * 32 < sg.m - mt * kTcSwRows)
                                  : hq < nacc * nblk;
            if (MODE != kTcGroupedSwiglu || duty) {
                if (!ok || !mbar_wait(acc_full + 16 * buf, use & 1, abort_flag, true)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
            }
            if (duty) {
                const int acc = hq / nblk, cb = hq - acc * nblk;
                const int row = MODE == kTcGroupedSwiglu ? mt * kTcSwRows + (q - 1) * 32 + lane
                                                         : mt * kTcRows + acc * 128 + q * 32 + lane;
                const bool whole = kc0 == 0 && kc1 == nkc;
                const uint32_t taddr = tmem + ((uint32_t) (q * 32) << 16) + (acc + buf) * 256 + cb * 128;
                const int col0 = nt * kTcCols + cb * 128;
                if constexpr (MODE == kTcGroupedSwiglu) {
                    // whole tiles only; rows past the expert's are not stored.  Image row
                    // irow: k chunk kc at kc * xt_rows * 128 bytes, 16-byte chunks swizzled
                    const int irow = sg.row0 + row;
                    uint8_t* rowp = row < sg.m ? a.img + ((size_t) irow * 128 + (size_t) (nt * 2) * a.xt_rows * 128)
                                               : nullptr;
                    const size_t kstride = (size_t) a.xt_rows * 128;
                    const int sw = irow & 7;
                    tc_epilogue_swiglu(taddr - cb * 128, cb, 1 + 2 * q, sg.svh + nt * 128, sg.svh2 + nt * 128,
                                       sg.suh2 + nt * 128, a.swiglu_limit, true, nullptr, false,
                                       [&](int col, uint4 v) {
                                           if (rowp)
                                               *reinterpret_cast<uint4*>(rowp + (col >> 6) * kstride +
                                                                         ((((col & 63) >> 3) ^ sw) << 4)) = v;
                                       });
                } else if constexpr (MODE == kTcDenseSwiglu) {
                    float* slot_row = nullptr;
                    if (!whole) {
                        const int slot = tc_cta_of(a.iters, nkc, grid, (long long) tile * nkc);
                        slot_row = a.slots + (size_t) slot * kTcSlotFloats + (size_t) (acc * 128 + q * 32 + lane) * kTcCols;
                    }
                    // the two warps (cb = role 0, 1) of this quarter share accumulator acc
                    uint8_t* img = a.img;
                    const int nkc2 = a.inter >> 6;
                    tc_epilogue_swiglu(taddr - cb * 128, cb, 1 + 2 * q + acc, a.svh + nt * 128,
                                       a.svh + a.inter + nt * 128, a.suh2 + nt * 128, a.swiglu_limit, whole,
                                       slot_row, row < a.m, [&](int col, uint4 v) {
                                           const int c = nt * 128 + col, rr = row & 127;
                                           *reinterpret_cast<uint4*>(
                                               img + ((((size_t) (row >> 7) * nkc2 + (c >> 6)) << 14) + rr * 128 +
                                                      ((((c & 63) >> 3) ^ (rr & 7)) << 4))) = v;
                                       });
                } else if constexpr (MODE == kTcDense) {
                    float* slot_row = nullptr;
                    if (!whole) {
                        const int slot = tc_cta_of(a.iters, nkc, grid, (long long) tile * nkc);
                        slot_row = a.slots + (size_t) slot * kTcSlotFloats +
                                   (size_t) (acc * 128 + q * 32 + lane) * kTcCols + cb * 128;
                    }
                    tc_epilogue_block(a, taddr, row, col0, whole, slot_row);
                } else if constexpr (MODE == kTcGroupedStore) {
                    float* dst = row < sg.m ? sg.gout + (size_t) row * a.out_stride + col0 : nullptr;
                    if (whole) tc_epilogue_block_grouped<true>(taddr, sg.svh + col0, dst, 1.f);
                    else tc_epilogue_block_grouped<false>(taddr, sg.svh + col0, dst, 1.f);
                } else {
                    float* dst = nullptr;
                    float w = 0.f;
                    if (row < sg.m) {
                        const int sl = sg.slot0 + row;
                        dst = reinterpret_cast<float*>(a.out) + (size_t) a.slot_token[sl] * a.out_stride + col0;
                        w = a.slot_weight[sl];
                    }
                    tc_epilogue_block_grouped<false>(taddr, sg.svh + col0, dst, w);
                }
            }
            tc_fence_before();
            __syncwarp();
            if constexpr (MODE == kTcGroupedSwiglu) {
                // 6 arrivals per phase: one per duty warp, the rest given by quarter 1's role-0
                // warp (always on duty); warps without duty never touch the barrier, so none can
                // arrive for a later use of the buffer before this phase completes
                if (duty && lane == 0) {
                    const int nq = min(3, (sg.m - mt * kTcSwRows + 31) >> 5);
                    mbar_arrive_n(acc_empty + 16 * buf, (q == 1 && hq == 0) ? 1u + (uint32_t) (6 - 2 * nq) : 1u);
                }
            } else {
                if (lane == 0) mbar_arrive(acc_empty + 16 * buf);
            }
            it += kc1 - kc0;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// CTA-pair matmul (dense modes, large M): a 2-CTA cluster computes 512 x 256 tiles
// with tcgen05.mma.cta_group::2 (M = 256 per MMA, two accumulators).  Each CTA holds
// two 128-row accumulators (pair rows 256 acc + 128 rank + [0, 128)) and decodes only
// its half of the tile's 256 B columns (rank 0: columns 0..127, rank 1: 128..255; the
// SwiGLU mode: gate block / up block), so every decoded code tile feeds 512 rows
// instead of 256 - half the decode work per output of the single-CTA kernel, at the
// same MMA work per SM.  Roles as in exl3_tc_gemm_kernel; warp 1 of the leader (rank
// 0) issues the MMAs, warp 1 of the other CTA forwards "stage full" (its own A copies
// and B decode done) to the leader's pfull barrier.  The leader's commits arrive on
// the empty and accumulator barriers of both CTAs (multicast); the epilogue warps of
// both CTAs arrive on the leader's acc_empty.  Every wait is bounded as in the
// single-CTA kernel.  All copies are unicast bulk copies into the issuing CTA's own
// shared memory (no multicast loads).
// ---------------------------------------------------------------------------
constexpr int kTpStages = 4;   // activation and B ring depth of the pair kernel
constexpr int kTpStagesT = 8;  // code ring depth of the pair kernel

template <int K>
struct TcPairSmem {
    static constexpr int kBars = 4 * kTpStages + 2 * kTpStagesT + kTpStages + 2;  // a, b, t; pfull; acc
    static constexpr uint32_t kBStage = 128 * 64 * 2;                // 16 KB: 128 columns x 64 k
    static constexpr uint32_t kTChunk = 4u * 8u * 32u * K;           // codes of 4 k-tiles x 8 n-tiles
    static constexpr uint32_t kA = 0;
    static constexpr uint32_t kB = kA + kTpStages * 2 * kTcABlock;
    static constexpr uint32_t kT = kB + kTpStages * kBStage;
    static constexpr uint32_t kBar = kT + kTpStagesT * kTChunk;
    static constexpr uint32_t kMisc = kBar + 8 * kBars;
    static constexpr uint32_t kBytes = kMisc + 16;
    static constexpr uint32_t kLaunchBytes = kBytes + 1024;
};

template <int K, int CB, int MODE>
__global__ __launch_bounds__(kTcThreads, 1) void exl3_tc_pair_kernel(const __grid_constant__ TcArgs a)
{
    static_assert(MODE == kTcDense || MODE == kTcDenseSwiglu, "pair tiles: dense modes");
    constexpr int S = kTpStages, ST = kTpStagesT;
    using L = TcPairSmem<K>;
    static_assert(L::kLaunchBytes <= 232448, "shared memory per CTA");
    extern __shared__ uint8_t tc_smem_raw[];
    const uint32_t raw = smem_u32(tc_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* gbase = tc_smem_raw + (base - raw);
    const uint32_t sA = base + L::kA, sB = base + L::kB, sT = base + L::kT, sBar = base + L::kBar;
    const uint32_t full_a = sBar, empty_a = full_a + 8 * S;
    const uint32_t full_t = empty_a + 8 * S, empty_t = full_t + 8 * ST;
    const uint32_t full_b = empty_t + 8 * ST, empty_b = full_b + 8 * S;
    const uint32_t pfull = empty_b + 8 * S;
    const uint32_t acc_full = pfull + 8 * S, acc_empty = acc_full + 8;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gbase + L::kMisc);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + L::kMisc + 4);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int npairs = gridDim.x >> 1;
    const int pair = blockIdx.x >> 1;
    const int nkc = a.nkc;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(full_a + 8 * i, 1);
            mbar_init(empty_a + 8 * i, 1);
            mbar_init(full_b + 8 * i, kTcDecWarps);
            mbar_init(empty_b + 8 * i, 1);
            mbar_init(pfull + 8 * i, 1);
        }
        for (int i = 0; i < ST; ++i) {
            mbar_init(full_t + 8 * i, 1);
            mbar_init(empty_t + 8 * i, kTcDecWarps);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * (kTcWarps - 3));  // every decoder and epilogue-only warp of both CTAs
        *abort_flag = 0;
        *reinterpret_cast<volatile unsigned long long*>(gbase + L::kMisc + 8) = a.wait_ns;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        tmem_alloc_pair(base + L::kMisc, 512);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    tc_griddep_launch();
    const TcRanges rg = tc_ranges(a.iters, nkc, npairs, pair);
    const int mpad = (a.m + 127) & ~127;

    if (warp == 0) {
        // activation producer: this CTA's two 128-row blocks of the pair tile
        tc_griddep_wait();
        if (lane == 0) {
            uint32_t s = 0, ph = 0, used = 0, par = 0;
            bool ok = true;
            for (int r = 0; r < 2; ++r)
            for (long long it = rg.b[r], it_end = rg.e[r]; it < it_end && ok;) {
                const int tile = (int) (it / nkc), kc0 = (int) (it - (long long) tile * nkc);
                const int kc1 = (int) min((long long) nkc, kc0 + (it_end - it));
                const int mt = tile % a.mtiles;
                const int blk0 = 4 * mt + (int) rank, blk1 = blk0 + 2;
                const bool has0 = blk0 * 128 < mpad, has1 = blk1 * 128 < mpad;
                const uint32_t bytes = (has0 ? kTcABlock : 0) + (has1 ? kTcABlock : 0);
                for (int kc = kc0; kc < kc1; ++kc) {
                    if (!mbar_wait(empty_a + 8 * s, ph ^ 1, abort_flag, true)) { ok = false; break; }
                    if (bytes) {
                        mbar_expect_tx(full_a + 8 * s, bytes);
                        if (has0) bulk_g2s(sA + (s * 2) * kTcABlock, a.xt + (((size_t) blk0 * nkc + kc) << 14), kTcABlock,
                                           full_a + 8 * s);
                        if (has1)
                            bulk_g2s(sA + (s * 2 + 1) * kTcABlock, a.xt + (((size_t) blk1 * nkc + kc) << 14), kTcABlock,
                                     full_a + 8 * s);
                        used |= 1u << s;
                        par = (par & ~(1u << s)) | (ph << s);
                    } else {
                        // nothing of this CTA's rows: the stage is ready as is.  Its last use
                        // now has no copy in flight, and the drain below must not wait on the
                        // parity of an older copy (the barrier may have wrapped back to it)
                        mbar_arrive(full_a + 8 * s);
                        used &= ~(1u << s);
                    }
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                it += kc1 - kc0;
            }
            for (uint32_t j = 0; j < S; ++j)
                if (used >> j & 1) mbar_wait(full_a + 8 * j, par >> j & 1, abort_flag, false);
        }
    } else if (warp == 2) {
        // code producer: this CTA's 8 n-tiles of each of the stage's 4 k-tile rows
        if (lane == 0) {
            const size_t row_bytes = (size_t) (a.n >> 4) * 32 * K;
            constexpr uint32_t seg = 8u * 32u * K;
            uint32_t s = 0, ph = 0, used = 0, par = 0;
            bool ok = true;
            for (int r = 0; r < 2; ++r)
            for (long long it = rg.b[r], it_end = rg.e[r]; it < it_end && ok;) {
                const int tile = (int) (it / nkc), kc0 = (int) (it - (long long) tile * nkc);
                const int kc1 = (int) min((long long) nkc, kc0 + (it_end - it));
                const int nt = tile / a.mtiles;
                // dense: columns 256 nt + 128 rank; swiglu: gate block nt (rank 0) or up block nt (rank 1)
                const size_t col_off = MODE == kTcDenseSwiglu
                                           ? ((size_t) nt * 8 + (size_t) rank * (a.inter >> 4)) * 32 * K
                                           : ((size_t) nt * 16 + (size_t) rank * 8) * 32 * K;
                const uint8_t* src = a.trellis + (size_t) kc0 * 4 * row_bytes + col_off;
                for (int kc = kc0; kc < kc1; ++kc, src += 4 * row_bytes) {
                    if (!mbar_wait(empty_t + 8 * s, ph ^ 1, abort_flag, true)) { ok = false; break; }
                    mbar_expect_tx(full_t + 8 * s, 4 * seg);
                    const uint32_t dst = sT + s * L::kTChunk;
#pragma unroll
                    for (int i = 0; i < 4; ++i) bulk_g2s(dst + i * seg, src + i * row_bytes, seg, full_t + 8 * s);
                    used |= 1u << s;
                    par = (par & ~(1u << s)) | (ph << s);
                    if (++s == ST) { s = 0; ph ^= 1; }
                }
                it += kc1 - kc0;
            }
            for (uint32_t j = 0; j < ST; ++j)
                if (used >> j & 1) mbar_wait(full_t + 8 * j, par >> j & 1, abort_flag, false);
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // MMA issuer (leader): both CTAs' stage s ready -> 8 pair MMAs
            uint32_t s = 0, ph = 0;
            int seg_i = 0;
            bool ok = true;
            const uint64_t a_desc0 = sw128_desc(sA), b_desc0 = sw128_desc(sB);
            const uint32_t idesc = tc_idesc(256, 256);
            for (int r = 0; r < 2; ++r)
            for (long long it = rg.b[r], it_end = rg.e[r]; it < it_end && ok; ++seg_i) {
                const int tile = (int) (it / nkc), kc0 = (int) (it - (long long) tile * nkc);
                const int kc1 = (int) min((long long) nkc, kc0 + (it_end - it));
                const int mt = tile % a.mtiles;
                const int nacc = a.m - mt * 512 > 256 ? 2 : 1;
                if (!mbar_wait_cl(acc_empty, (uint32_t) (seg_i & 1) ^ 1, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kc = kc0; kc < kc1; ++kc) {
                    // the other CTA's arrival on pfull is a cluster-scope release: acquire at cluster scope
                    if (!mbar_wait(full_a + 8 * s, ph, abort_flag, true) || !mbar_wait(full_b + 8 * s, ph, abort_flag, true) ||
                        !mbar_wait_cl(pfull + 8 * s, ph, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = a_desc0 + s * (2 * kTcABlock >> 4);
                    const uint64_t bd = b_desc0 + s * (L::kBStage >> 4);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint32_t acc_flag = (kc != kc0 || ks != 0) ? 1u : 0u;
                        tc_mma_pair(tmem, ad + 2 * ks, bd + 2 * ks, idesc, acc_flag);
                        if (nacc == 2) tc_mma_pair(tmem + 256, ad + (kTcABlock >> 4) + 2 * ks, bd + 2 * ks, idesc, acc_flag);
                    }
                    tc_commit_pair(empty_a + 8 * s);
                    tc_commit_pair(empty_b + 8 * s);
                    if (++s == S) { s = 0; ph ^= 1; }
                }
                tc_commit_pair(acc_full);
                it += kc1 - kc0;
            }
            if (seg_i > 0) mbar_wait(acc_full, (uint32_t) ((seg_i - 1) & 1), abort_flag, false);
        } else if (lane == 0) {
            // forwarder (rank 1): this CTA's A blocks and B half of stage s are in place
            const uint32_t remote_pfull = mapa_shared(pfull, 0);
            uint32_t s = 0, ph = 0;
            bool ok = true;
            for (int r = 0; r < 2; ++r)
            for (long long it = rg.b[r], it_end = rg.e[r]; it < it_end && ok; ++it) {
                if (!mbar_wait(full_a + 8 * s, ph, abort_flag, true) || !mbar_wait(full_b + 8 * s, ph, abort_flag, true)) {
                    ok = false;
                    break;
                }
                mbar_arrive_cluster(remote_pfull + 8 * s);
                if (++s == S) { s = 0; ph ^= 1; }
            }
        }
    } else {
        // decoders (and the epilogue of their TMEM lane quarter) or epilogue-only warps
        const int q = warp & 3;
        const int hq = q == 3 ? warp >> 2 : (warp >> 2) - 1;
        const bool decoder = q != 1;
        const int dw = (warp - 3) - (warp - 2) / 4;
        const uint32_t acc_empty_leader = mapa_shared(acc_empty, 0);

        tc_griddep_wait();
        const LaneWords lw = lane_words<K>(lane);
        uint32_t st = 0, pt = 0, sb = 0, pb = 0;
        int seg_i = 0;
        bool ok = true;
        for (int r = 0; r < 2; ++r)
        for (long long it = rg.b[r], it_end = rg.e[r]; it < it_end && ok; ++seg_i) {
            const int tile = (int) (it / nkc), kc0 = (int) (it - (long long) tile * nkc);
            const int kc1 = (int) min((long long) nkc, kc0 + (it_end - it));
            const int mt = tile % a.mtiles, nt = tile / a.mtiles;
            if (decoder) {
                for (int kc = kc0; kc < kc1; ++kc) {
                    if (!mbar_wait(full_t + 8 * st, pt, abort_flag, true) ||
                        !mbar_wait(empty_b + 8 * sb, pb ^ 1, abort_flag, true)) {
                        ok = false;
                        break;
                    }
                    tc_decode_stage<K, CB, 8>(sT + st * L::kTChunk, sB + sb * L::kBStage, dw, lane, lw);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(full_b + 8 * sb);
                        mbar_arrive(empty_t + 8 * st);
                    }
                    if (++st == ST) { st = 0; pt ^= 1; }
                    if (++sb == S) { sb = 0; pb ^= 1; }
                }
            }
            if (!ok || !mbar_wait(acc_full, (uint32_t) (seg_i & 1), abort_flag, true)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const int nacc = a.m - mt * 512 > 256 ? 2 : 1;
            if (hq < 2 * nacc) {
                const int acc = hq >> 1, cb = hq & 1;
                const int srow = acc * 128 + q * 32 + lane;  // row of this CTA's accumulators (and slot)
                const int row = mt * 512 + acc * 256 + (int) rank * 128 + q * 32 + lane;
                const bool whole = kc0 == 0 && kc1 == nkc;
                const uint32_t taddr = tmem + ((uint32_t) (q * 32) << 16) + acc * 256 + cb * 128;
                float* slot_row = nullptr;
                if (!whole) {
                    const int slot = 2 * tc_cta_of(a.iters, nkc, npairs, (long long) tile * nkc) + (int) rank;
                    slot_row = a.slots + (size_t) slot * kTcSlotFloats + (size_t) srow * kTcCols;
                }
                if constexpr (MODE == kTcDenseSwiglu) {
                    uint8_t* img = a.img;
                    const int nkc2 = a.inter >> 6;
                    const bool row_ok = row < a.m;
                    tc_epilogue_swiglu(taddr - cb * 128, cb, 1 + 2 * q + acc, a.svh + nt * 128,
                                       a.svh + a.inter + nt * 128, a.suh2 + nt * 128, a.swiglu_limit, whole,
                                       slot_row, row_ok, [&](int col, uint4 v) {
                                           if (!row_ok) return;
                                           const int c = nt * 128 + col, rr = row & 127;
                                           *reinterpret_cast<uint4*>(
                                               img + ((((size_t) (row >> 7) * nkc2 + (c >> 6)) << 14) + rr * 128 +
                                                      ((((c & 63) >> 3) ^ (rr & 7)) << 4))) = v;
                                       });
                } else {
                    tc_epilogue_block(a, taddr, row, nt * kTcCols + cb * 128, whole, slot_row ? slot_row + cb * 128 : nullptr);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (rank == 0) mbar_arrive(acc_empty);
                else mbar_arrive_cluster(acc_empty_leader);
            }
            it += kc1 - kc0;
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // the leader's MMAs into this CTA's TMEM are complete
    if (warp == 0) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc_pair(tmem, 512);
    }
}

// Split tiles: the slot of CTA c holds the tile that contains the end of c's
// stream-K range, when that tile starts inside the range.  One CTA per slot.
// Slot row sr of CTA c's split tile -> row of the output (or -1 past m).  Single-CTA
// tiles: 256 rows, slot row = tile row; pair tiles: 512 rows, the slot holds the CTA's
// two 128-row accumulators (pair rows 256 acc + 128 rank + [0, 128)).
__device__ __forceinline__ int tc_slot_row(const TcArgs& a, int c, int mt, int sr)
{
    const int row = a.pair ? mt * 512 + (sr >> 7) * 256 + (c & 1) * 128 + (sr & 127) : mt * kTcRows + sr;
    return row < a.m ? row : -1;
}

// The split tile whose partial sums CTA c's slot holds, or -1.
__device__ __forceinline__ int tc_slot_tile(const TcArgs& a, int c, int grid)
{
    const TcRanges rg = a.pair ? tc_ranges(a.iters, a.nkc, grid >> 1, c >> 1) : tc_ranges(a.iters, a.nkc, grid, c);
    const long long start = rg.b[1];
    const long long end = rg.e[1];
    if (end >= a.iters || end % a.nkc == 0) return -1;
    const int tile = (int) (end / a.nkc);
    if ((long long) tile * a.nkc < start) return -1;
    return tile;
}

__global__ __launch_bounds__(256) void exl3_tc_finish_kernel(const __grid_constant__ TcArgs a, int grid)
{
    tc_griddep_wait();
    const int c = blockIdx.x;
    const int tile = tc_slot_tile(a, c, grid);
    if (tile < 0) return;
    const int mt = tile % a.mtiles, nt = tile / a.mtiles;
    const int cols = min(kTcCols, a.n - nt * kTcCols);
    float* slot = a.slots + (size_t) c * kTcSlotFloats;
    const int cols8 = cols >> 3;
    for (int e = threadIdx.x; e < kTcRows * cols8; e += blockDim.x) {
        const int r = e / cols8, c8 = (e - r * cols8) * 8;
        const int row = tc_slot_row(a, c, mt, r);
        if (row < 0) continue;  // never written: still zero
        float4* src = reinterpret_cast<float4*>(slot + (size_t) r * kTcCols + c8);
        const float4 p0 = __ldcg(src), p1 = __ldcg(src + 1);
        __stcg(src, make_float4(0.f, 0.f, 0.f, 0.f));
        __stcg(src + 1, make_float4(0.f, 0.f, 0.f, 0.f));
        const float v[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
        store8(a, row, nt * kTcCols + c8, v);
    }
}

// Split tiles of a SwiGLU launch: the slot row holds y of the gate block (columns
// 0..127) and of the up block (128..255); one warp per row completes the epilogue
// of tc_epilogue_swiglu (lane holds columns lane + 32 i) and re-zeroes the slot.
__global__ __launch_bounds__(256) void exl3_tc_finish_swiglu_kernel(const __grid_constant__ TcArgs a, int grid)
{
    tc_griddep_wait();
    const int c = blockIdx.x;
    const int tile = tc_slot_tile(a, c, grid);
    if (tile < 0) return;
    const int mt = tile % a.mtiles, nt = tile / a.mtiles;
    const int lane = threadIdx.x & 31;
    const int nkc2 = a.inter >> 6;
    float* slot = a.slots + (size_t) c * kTcSlotFloats;
    for (int r = threadIdx.x >> 5; r < kTcRows; r += blockDim.x >> 5) {
        const int row = tc_slot_row(a, c, mt, r);
        if (row < 0) continue;  // never written: still zero
        float* sr = slot + (size_t) r * kTcCols;
        float v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int col = lane + 32 * i;
            const float g = __ldcg(sr + col), u = __ldcg(sr + 128 + col);
            __stcg(sr + col, 0.f);
            __stcg(sr + 128 + col, 0.f);
            v[i] = swiglu_pre(g, u, a.swiglu_limit, __half2float(a.suh2[nt * 128 + col]));
        }
        warp_fwht128(v, lane);
        const int rr = row & 127;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int col = nt * 128 + lane + 32 * i;
            uint8_t* dst = a.img + ((((size_t) (row >> 7) * nkc2 + (col >> 6)) << 14) + rr * 128 +
                                    ((((col & 63) >> 3) ^ (rr & 7)) << 4) + (col & 7) * 2);
            *reinterpret_cast<__half*>(dst) = __float2half_rn(__fmul_rn(v[i], kHadScale));
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
static int tc_sm_count()
{
    static int count[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!count[dev]) {
        int c = 0;
        if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0) c = 148;
        count[dev] = c;
    }
    return count[dev];
}

static cudaError_t tc_launch(const void* kern, int grid, int block, size_t smem, cudaStream_t stream, void** args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) grid);
    cfg.blockDim = dim3((unsigned) block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, kern, args);
}

// The CTA-pair kernel: clusters of 2 CTAs, programmatic dependent launch.
template <int K, int CB, int MODE>
static int tc_launch_pair(const TcArgs& a, int grid, cudaStream_t stream)
{
    using L = TcPairSmem<K>;
    static bool configured[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kErrLaunch;
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(exl3_tc_pair_kernel<K, CB, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int) L::kLaunchBytes) != cudaSuccess)
            return kErrLaunch;
        configured[dev] = true;
    }
    TcArgs arg = a;
    arg.wait_ns = wait_limit_ns(kTcTimeoutNs);
    void* args[] = {&arg};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) grid);
    cfg.blockDim = dim3((unsigned) kTcThreads);
    cfg.dynamicSmemBytes = L::kLaunchBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelExC(&cfg, (const void*) exl3_tc_pair_kernel<K, CB, MODE>, args) == cudaSuccess ? kOk
                                                                                                          : kErrLaunch;
}

template <int MODE>
static int tc_launch_pair_k(const TcArgs& a, int K, int cb, int grid, cudaStream_t stream)
{
    switch (K * 4 + cb) {
        case 8: return tc_launch_pair<2, 0, MODE>(a, grid, stream);
        case 9: return tc_launch_pair<2, 1, MODE>(a, grid, stream);
        case 10: return tc_launch_pair<2, 2, MODE>(a, grid, stream);
        case 12: return tc_launch_pair<3, 0, MODE>(a, grid, stream);
        case 13: return tc_launch_pair<3, 1, MODE>(a, grid, stream);
        case 14: return tc_launch_pair<3, 2, MODE>(a, grid, stream);
        case 16: return tc_launch_pair<4, 0, MODE>(a, grid, stream);
        case 17: return tc_launch_pair<4, 1, MODE>(a, grid, stream);
        default: return tc_launch_pair<4, 2, MODE>(a, grid, stream);
    }
}

template <int K, int CB, int MODE>
static int tc_launch_gemm(const TcArgs& a, int grid, cudaStream_t stream)
{
    using L = TcSmem<K>;
    static bool configured[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return kErrLaunch;
    if (!configured[dev]) {
        if (cudaFuncSetAttribute(exl3_tc_gemm_kernel<K, CB, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int) L::kLaunchBytes) != cudaSuccess)
            return kErrLaunch;
        configured[dev] = true;
    }
    TcArgs arg = a;
    arg.wait_ns = wait_limit_ns(kTcTimeoutNs);
    void* args[] = {&arg};
    return tc_launch((const void*) exl3_tc_gemm_kernel<K, CB, MODE>, grid, kTcThreads, L::kLaunchBytes, stream,
                     args) == cudaSuccess
               ? kOk
               : kErrLaunch;
}

template <int K, int MODE>
static int tc_launch_cb(const TcArgs& a, int cb, int grid, cudaStream_t stream)
{
    if (cb == 0) return tc_launch_gemm<K, 0, MODE>(a, grid, stream);
    if (cb == 1) return tc_launch_gemm<K, 1, MODE>(a, grid, stream);
    return tc_launch_gemm<K, 2, MODE>(a, grid, stream);
}

template <int MODE>
static int tc_launch_k(const TcArgs& a, int K, int cb, int grid, cudaStream_t stream)
{
    switch (K) {
        case 2: return tc_launch_cb<2, MODE>(a, cb, grid, stream);
        case 3: return tc_launch_cb<3, MODE>(a, cb, grid, stream);
        default: return tc_launch_cb<4, MODE>(a, cb, grid, stream);
    }
}

int tc_device_sms() { return tc_sm_count(); }

int tc_grouped_matmul(const TcGroupedCall& c, int K, int cb, cudaStream_t stream)
{
    if (K < 2 || K > 4) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (c.k <= 0 || c.n <= 0 || c.k % 128 || c.n % 128 || c.xt_rows % 8 || c.out_stride % 4) return kErrBadShape;
    if (!c.probs || !c.tile_prob || !c.dev_tiles) return kErrNullPointer;
    if (c.mode == kTcGroupedSwiglu ? !c.img : !c.out) return kErrNullPointer;
    if (c.mode == kTcGroupedCombine && (!c.slot_token || !c.slot_weight)) return kErrNullPointer;
    TcArgs a = {};
    a.out = c.out;
    a.out_stride = c.out_stride;
    a.k = c.k;
    a.n = c.n;
    a.nkc = c.k / 64;
    a.out_dtype = 2;
    a.probs = c.probs;
    a.tile_prob = c.tile_prob;
    a.dev_tiles = c.dev_tiles;
    a.dev_tile_base = c.dev_tile_base;
    a.xt_rows = c.xt_rows;
    a.slot_token = c.slot_token;
    a.slot_weight = c.slot_weight;
    a.img = c.img;
    a.swiglu_limit = c.swiglu_limit;
    a.inter = c.n;
    const int grid = tc_sm_count();  // the tile count is known on the device only
    if (c.mode == kTcGroupedSwiglu) return tc_launch_k<kTcGroupedSwiglu>(a, K, cb, grid, stream);
    if (c.mode == kTcGroupedStore) return tc_launch_k<kTcGroupedStore>(a, K, cb, grid, stream);
    if (c.mode == kTcGroupedCombine) return tc_launch_k<kTcGroupedCombine>(a, K, cb, grid, stream);
    return kErrBadArgument;
}

size_t tc_xt_bytes(int m, int k) { return (size_t) ((m + 127) / 128) * 128 * (size_t) k * 2; }

size_t tc_state_bytes() { return (size_t) tc_sm_count() * kTcSlotFloats * sizeof(float); }

// One dense tensor-core matmul: the input stage (x -> image, unless the image was
// written by an earlier kernel), the GEMM (plain epilogue, or the SwiGLU epilogue that
// writes the down projection's image), and the kernel finishing split tiles.
int tc_dense_run(const TcDenseRun& r, cudaStream_t st)
{
    const bool swiglu = r.img != nullptr;
    // CTA pairs (512-row tiles) where they measured faster: the SwiGLU gate|up from
    // kTcPairMinRows rows; plain GEMMs from kTcPairDenseMinRows rows with a long k (every
    // 256-column tile whole)
    const bool auto_pair = swiglu ? r.m >= kTcPairMinRows : (r.m >= kTcPairDenseMinRows && r.k >= kTcPairDenseMinK);
    const bool pair = r.pair != 0 && (r.pair > 0 || auto_pair) && (swiglu || r.n % kTcCols == 0) && tc_sm_count() >= 2;
    const int mtiles = pair ? (r.m + 511) / 512 : (r.m + kTcRows - 1) / kTcRows;
    const int ntiles = swiglu ? r.n / 256 : (r.n + kTcCols - 1) / kTcCols;
    const long long tiles = (long long) mtiles * ntiles;
    if (tiles > 0x7fffffffLL) return kErrBadShape;
    const int nkc = r.k / 64;
    const long long iters = tiles * nkc;
    const int grid = pair ? 2 * (int) std::min<long long>(tc_sm_count() / 2, iters)
                          : (int) std::min<long long>(tc_sm_count(), iters);

    if (r.run_input) {
        const int mpad = (r.m + 127) / 128 * 128;
        const int in_tasks = mpad * (r.k / 128);
        const int in_grid = std::min((in_tasks + 7) / 8, 8 * tc_sm_count());
        exl3_tc_input_kernel<<<in_grid, 256, 0, st>>>(reinterpret_cast<const __half*>(r.x), r.x_stride, r.suh, r.m,
                                                       mpad, r.k, r.xt);
        if (cudaPeekAtLastError() != cudaSuccess) return kErrLaunch;
    }

    TcArgs a = {};
    a.xt = r.xt;
    a.trellis = reinterpret_cast<const uint8_t*>(r.trellis);
    a.svh = r.svh;
    a.out = r.out;
    a.slots = r.slots;
    a.out_stride = r.out_stride;
    a.iters = iters;
    a.m = r.m;
    a.k = r.k;
    a.n = r.n;
    a.mtiles = mtiles;
    a.tiles = (int) tiles;
    a.nkc = nkc;
    a.out_dtype = r.out_dtype;
    const int esz = r.out_dtype == 2 ? 4 : 2;
    a.vec_store = r.out && ((uintptr_t) r.out % 16 == 0) && ((r.out_stride * esz) % 16 == 0);
    a.img = r.img;
    a.suh2 = r.suh2;
    a.swiglu_limit = r.swiglu_limit;
    a.inter = r.n / 2;
    a.pair = pair ? 1 : 0;
    int rc;
    if (pair)
        rc = swiglu ? tc_launch_pair_k<kTcDenseSwiglu>(a, r.K, r.cb, grid, st)
                    : tc_launch_pair_k<kTcDense>(a, r.K, r.cb, grid, st);
    else
        rc = swiglu ? tc_launch_k<kTcDenseSwiglu>(a, r.K, r.cb, grid, st) : tc_launch_k<kTcDense>(a, r.K, r.cb, grid, st);
    if (rc != kOk) return rc;
    if (grid > (pair ? 2 : 1)) {
        int g = grid;
        void* args[] = {&a, &g};
        const void* fin = swiglu ? (const void*) exl3_tc_finish_swiglu_kernel : (const void*) exl3_tc_finish_kernel;
        if (tc_launch(fin, grid, 256, 0, st, args) != cudaSuccess) return kErrLaunch;
    }
    return kOk;
}

}  // namespace exl3b200

using namespace exl3b200;

extern "C" size_t exl3b200_gemm_scratch_size(int m, int k)
{
    if (m <= 0 || k <= 0 || k % 128) return 0;
    return tc_xt_bytes(m, k);
}

extern "C" size_t exl3b200_gemm_state_size(void) { return tc_state_bytes(); }

extern "C" int exl3b200_gemm(const void* x, long long x_stride, int m, int k, const void* trellis, int n, int K, int cb,
                             const void* suh, const void* svh, void* out, long long out_stride, int out_dtype,
                             int flags, void* state, size_t state_bytes, void* scratch, size_t scratch_bytes,
                             void* stream)
{
    if (!x || !out || !trellis || !svh || !scratch || !state) return kErrNullPointer;
    if (K < 2 || K > 4) return kErrBadBits;
    if (cb < 0 || cb > 2) return kErrBadCodebook;
    if (out_dtype < 0 || out_dtype > 2) return kErrBadArgument;
    if (m < 1 || k <= 0 || n <= 0 || (k % 128) || (n % 128)) return kErrBadShape;
    if (x_stride < k || out_stride < n) return kErrBadShape;
    const bool pre_rotated = (flags & EXL3B200_FLAG_INPUT_ROTATED) != 0;
    if (!pre_rotated && !suh) return kErrNullPointer;
    if (((uintptr_t) x & 1) || ((uintptr_t) out & 3)) return kErrUnaligned;
    if (((uintptr_t) trellis & 15) || ((uintptr_t) scratch & 15) || ((uintptr_t) svh & 15)) return kErrUnaligned;
    if ((uintptr_t) state & 15) return kErrUnaligned;
    if (scratch_bytes < tc_xt_bytes(m, k) || state_bytes < tc_state_bytes()) return kErrWorkspace;
    TcDenseRun r = {};
    r.pair = (flags & EXL3B200_FLAG_SINGLE_CTA) ? 0 : (flags & EXL3B200_FLAG_PAIR_CTA) ? 1 : -1;
    r.x = x;
    r.x_stride = x_stride;
    r.suh = pre_rotated ? nullptr : reinterpret_cast<const __half*>(suh);
    r.run_input = true;
    r.xt = reinterpret_cast<uint8_t*>(scratch);
    r.trellis = trellis;
    r.svh = reinterpret_cast<const __half*>(svh);
    r.m = m;
    r.k = k;
    r.n = n;
    r.K = K;
    r.cb = cb;
    r.out = out;
    r.out_stride = out_stride;
    r.out_dtype = out_dtype;
    r.slots = reinterpret_cast<float*>(state);
    return tc_dense_run(r, reinterpret_cast<cudaStream_t>(stream));
}

namespace exl3b200 {
// Device address of the sticky status, for the kernels of other translation units.
int* exl3_status_dev_ptr()
{
    static int* cache[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!cache[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_exl3_device_status) != cudaSuccess) return nullptr;
        cache[dev] = reinterpret_cast<int*>(p);
    }
    return cache[dev];
}
}  // namespace exl3b200

extern "C" int exl3b200_device_status(int* host_status, int reset, void* stream)
{
    if (!host_status) return kErrNullPointer;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (cudaMemcpyFromSymbolAsync(host_status, g_exl3_device_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st) !=
        cudaSuccess)
        return kErrLaunch;
    if (reset) {
        static const int zero = 0;
        if (cudaMemcpyToSymbolAsync(g_exl3_device_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st) !=
            cudaSuccess)
            return kErrLaunch;
    }
    return kOk;
}
