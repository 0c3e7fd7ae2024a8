// Shared device helpers for the EXL3 B200 kernels: trellis window extraction,
// the three procedural codebooks, tensor-core fragment packing, the 128-point
// Walsh-Hadamard transform over one warp, and the status codes of the C ABI.
//
// EXL3 tile format (reference: csrc/exl3_dequant.cuh:110-135,
// csrc/quant/exl3_dq.cuh:15-31): a 16x16 weight tile is 16*K int16 words.  The
// words pair into little-endian uint32 words that form a cyclic bit stream read
// most-significant-bit first.  Element t (0..255) of the tile is the codebook
// entry of the 16-bit window ending at stream bit (t+1)*K-1 (mod 256*K).  Lane
// L of a warp owns elements t = 8L..8L+7, and element (L, j) sits at row
// k = 2(L%4) + (j&1) + 8((j>>1)&1), column n = L/4 + 8(j>>2) of the tile
// (reference: csrc/bindings.cpp:51-75) - exactly the A-operand fragment of an
// m16n8k16 MMA when the tile is used transposed (rows = n, cols = k).
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace exl3b200 {

// ---------------------------------------------------------------------------
// status codes (mirrored in include/exl3_b200.h)
// ---------------------------------------------------------------------------
enum Status : int {
    kOk = 0,
    kErrBadShape = 1,
    kErrBadBits = 2,
    kErrBadCodebook = 3,
    kErrUnaligned = 4,
    kErrLaunch = 5,
    kErrWorkspace = 6,
    kErrNullPointer = 7,
    kErrBadArgument = 8,
    kErrTimeout = 9,
};

constexpr uint32_t kInst3Mult = 89226354u;
constexpr uint32_t kInst3Add = 64248484u;
constexpr uint32_t kMcgMult = 0xCBAC1FEDu;
constexpr uint32_t kMul1Mult = 0x83DCD12Du;
constexpr uint16_t kMul1InvBits = 0x1EEE;   // fp16 0.00677
constexpr uint16_t kMul1BiasBits = 0xC931;  // fp16 -10.39
constexpr float kHadScale = 0.08838834764831845f;  // 1/sqrt(128)

__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t x)
{
    // (x & 0x8fff8fff) ^ 0x3b603b60 in one LOP3 (truth table 0x6a)
    uint32_t r;
    asm("lop3.b32 %0, %1, 0x8fff8fff, 0x3b603b60, 0x6a;" : "=r"(r) : "r"(x));
    return r;
}

__device__ __forceinline__ uint32_t dp4a_bytesum(uint32_t x, uint32_t acc)
{
    uint32_t r;
    asm("dp4a.u32.u32 %0, %1, 0x01010101, %2;" : "=r"(r) : "r"(x), "r"(acc));
    return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// Codebook "pre-value": the 32-bit word whose halves (cb 0/1) or low half (cb 2)
// carry the codebook entry of window w, before the final fp16 add / fma.
template <int CB>
__device__ __forceinline__ uint32_t codebook_pre(uint32_t w)
{
    if constexpr (CB == 0) return lop3_and_xor(w * kInst3Mult + kInst3Add);
    else if constexpr (CB == 1) return lop3_and_xor(w * kMcgMult);
    else return dp4a_bytesum(w * kMul1Mult, 0x6400u);   // fp16 bits of 1024 + bytesum
}

// Codebook entry as float, rounded to fp16 exactly as the device decode of the
// reference (__hadd / __hfma round to nearest, csrc/quant/codebook.cuh:56-90).
// cb 0/1: both halves have exponents 12..15, so the float sum is exact and the
// conversion is the single rounding.  cb 2: h*k_inv + k_bias is exact in float
// (22 significant bits), so again one rounding.
template <int CB>
__device__ __forceinline__ float codebook_value_rn(uint32_t w)
{
    const uint32_t p = codebook_pre<CB>(w);
    if constexpr (CB == 2) {
        const float h = __half2float(__ushort_as_half((uint16_t) (p & 0xffff)));
        const float v = __fmaf_rn(h, __half2float(__ushort_as_half(kMul1InvBits)),
                                  __half2float(__ushort_as_half(kMul1BiasBits)));
        return __half2float(__float2half_rn(v));
    } else {
        const float lo = __half2float(__ushort_as_half((uint16_t) (p & 0xffff)));
        const float hi = __half2float(__ushort_as_half((uint16_t) (p >> 16)));
        return __half2float(__float2half_rn(__fadd_rn(lo, hi)));
    }
}

// float -> fp16 by truncation, bit-compatible with the reference CPU helper
// float_to_half_bits (csrc/exl3_dequant.cuh:41-55), subnormal branch included.
__device__ __forceinline__ uint16_t trunc_half_bits(float v)
{
    const uint32_t raw = __float_as_uint(v);
    const uint32_t sign = (raw >> 16) & 0x8000u;
    const int e = (int) ((raw >> 23) & 0xffu) - 127;
    const uint32_t mant = raw & 0x7fffffu;
    if (e > 15) return (uint16_t) (sign | 0x7c00u);
    if (e < -14) {
        if (e < -24) return (uint16_t) sign;
        const uint32_t m = (mant | 0x800000u) >> (-e - 1);
        return (uint16_t) (sign | (m >> 13));
    }
    return (uint16_t) (sign | ((uint32_t) (e + 15) << 10) | (mant >> 13));
}

// Codebook entry with the reference CPU decode's truncating fp16 rounding
// (csrc/exl3_dequant.cuh:57-93): float add / mul+add, then truncation.
template <int CB>
__device__ __forceinline__ float codebook_value_trunc(uint32_t w)
{
    const uint32_t p = codebook_pre<CB>(w);
    float v;
    if constexpr (CB == 2) {
        const float h = __half2float(__ushort_as_half((uint16_t) (p & 0xffff)));
        v = __fadd_rn(__fmul_rn(h, __half2float(__ushort_as_half(kMul1InvBits))),
                      __half2float(__ushort_as_half(kMul1BiasBits)));
    } else {
        v = __fadd_rn(__half2float(__ushort_as_half((uint16_t) (p & 0xffff))),
                      __half2float(__ushort_as_half((uint16_t) (p >> 16))));
    }
    return __half2float(__ushort_as_half(trunc_half_bits(v)));
}

// ---------------------------------------------------------------------------
// trellis windows
// ---------------------------------------------------------------------------

// Window of tile element t from the tile's uint32 words (any K in 1..8).
template <int K>
__device__ __forceinline__ uint32_t tile_window(const uint32_t* words, int t)
{
    constexpr int n32 = 8 * K;
    const int b0 = ((t + 257) * K - 16) % (256 * K);
    const int i1u = (b0 + 15) >> 5;
    const int i0 = (b0 >> 5) % n32;
    const int i1 = i1u % n32;
    const int shift = (i1u + 1) * 32 - (b0 + 16);
    const uint64_t merged = ((uint64_t) words[i0] << 32) | (uint64_t) words[i1];
    return (uint32_t) (merged >> shift) & 0xffffu;
}

// Per-lane extraction constants for K <= 4, where the 8 windows of lane L lie
// inside two consecutive stream words wa, wb (wb = wa + 1 mod 8K, or wb = wa).
struct LaneWords {
    int wa;      // index of the first word
    int wb;      // index of the second word
    int shift7;  // right shift of the 64-bit (wa:wb) pair that yields window j = 7
};

template <int K>
__device__ __forceinline__ LaneWords lane_words(int lane)
{
    static_assert(K >= 1 && K <= 4, "two-word extraction needs K <= 4");
    constexpr int n32 = 8 * K;
    const int first = (8 * lane + 257) * K - 16;   // unwrapped start bit of window 0
    const int last = (8 * lane + 8 + 256) * K - 1;  // unwrapped end bit of window 7
    LaneWords lw;
    lw.wa = (first >> 5) % n32;
    lw.wb = (last >> 5) % n32;
    lw.shift7 = ((last >> 5) + 1) * 32 - 1 - last;
    if ((first >> 5) == (last >> 5)) lw.wa = lw.wb;  // all 8 windows inside one word
    return lw;
}

// Clean 16-bit window at bit offset off (0..16) of v: shift it to the top, then
// take the top half with one byte permute.  The left shift can issue on the FMA
// pipe (IMAD.SHL), which keeps the integer-logic pipe (half rate on sm_100) free.
template <int OFF>
__device__ __forceinline__ uint32_t win_at(uint32_t v)
{
    static_assert(OFF >= 0 && OFF <= 16, "window offset");
    if constexpr (OFF == 0) return v & 0xffffu;
    else if constexpr (OFF == 8) return prmt(v, 0u, 0x4421);
    else if constexpr (OFF == 16) return prmt(v, 0u, 0x4432);
    else return prmt(v << (16 - OFF), 0u, 0x4432);
}

__device__ __forceinline__ uint32_t win_at_rt(uint32_t v, uint32_t mul)
{
    // mul = 2^(16 - off), a per-lane constant
    return prmt(v * mul, 0u, 0x4432);
}

// The 8 windows of a lane (j = 0..7) from its two words a (earlier in the
// stream) and b.  Window j sits at offset shift7 + (7-j)*K of the 64-bit (a:b).
template <int K>
__device__ __forceinline__ void lane_windows(uint32_t a, uint32_t b, int shift7, uint32_t (&w)[8])
{
    if constexpr (K == 4) {
        // shift7 is 0 for every lane; offsets 0,4,...,28
        const uint32_t c = __funnelshift_r(b, a, 16);  // bits 16..47 of (a:b)
        w[7] = win_at<0>(b);
        w[6] = win_at<4>(b);
        w[5] = win_at<8>(b);
        w[4] = win_at<12>(b);
        w[3] = win_at<16>(b);
        w[2] = win_at<4>(c);
        w[1] = win_at<8>(c);
        w[0] = win_at<12>(c);
    } else if constexpr (K == 2) {
        // shift7 in {0, 16}; offsets shift7 + 0,2,...,14
        const uint32_t v = __funnelshift_r(b, a, shift7);
        w[7] = win_at<0>(v);
        w[6] = win_at<2>(v);
        w[5] = win_at<4>(v);
        w[4] = win_at<6>(v);
        w[3] = win_at<8>(v);
        w[2] = win_at<10>(v);
        w[1] = win_at<12>(v);
        w[0] = win_at<14>(v);
    } else if constexpr (K == 3) {
        // shift7 in 0..31 per lane; offsets shift7 + 0,3,...,21 (<= 52)
        const uint64_t pr = ((uint64_t) a << 32) | (uint64_t) b;
        const uint64_t t = pr >> shift7;
        const uint32_t v0 = (uint32_t) t;
        const uint32_t v1 = __funnelshift_r(v0, (uint32_t) (t >> 32), 16);  // offsets 16..47
        w[7] = win_at<0>(v0);
        w[6] = win_at<3>(v0);
        w[5] = win_at<6>(v0);
        w[4] = win_at<9>(v0);
        w[3] = win_at<12>(v0);
        w[2] = win_at<15>(v0);
        w[1] = win_at<2>(v1);
        w[0] = win_at<5>(v1);
    } else {
        const uint64_t v = ((uint64_t) a << 32) | (uint64_t) b;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            w[j] = (uint32_t) (v >> (shift7 + (7 - j) * K)) & 0xffffu;
    }
}

// ---------------------------------------------------------------------------
// 128-point Walsh-Hadamard transform over one warp.  Lane l holds elements
// l, l+32, l+64, l+96 in v[0..3]; butterflies run in the order of the sequential
// transform (strides 1, 2, 4, ..., 64; reference csrc/exl3_dequant.cuh:137-148),
// each output computed as a+b or a-b with a the lower-index input, so the float
// result is bit-identical to the sequential loop.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void warp_fwht128(float (&v)[4], int lane)
{
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const bool upper = (lane & m) != 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float peer = __shfl_xor_sync(0xffffffffu, v[i], m);
            v[i] = upper ? __fsub_rn(peer, v[i]) : __fadd_rn(v[i], peer);
        }
    }
    // stride 32: (l, l+32) and (l+64, l+96)
    {
        const float a0 = v[0], b0 = v[1], a1 = v[2], b1 = v[3];
        v[0] = __fadd_rn(a0, b0);
        v[1] = __fsub_rn(a0, b0);
        v[2] = __fadd_rn(a1, b1);
        v[3] = __fsub_rn(a1, b1);
    }
    // stride 64: (l, l+64) and (l+32, l+96)
    {
        const float a0 = v[0], b0 = v[2], a1 = v[1], b1 = v[3];
        v[0] = __fadd_rn(a0, b0);
        v[2] = __fsub_rn(a0, b0);
        v[1] = __fadd_rn(a1, b1);
        v[3] = __fsub_rn(a1, b1);
    }
}

// fp16 H128(x * suh) / sqrt(128) of one 128-block over a warp, with the
// reference's roundings (had_hf_r_128_inner<true,false>,
// csrc/quant/hadamard_inner.cuh:93-147): fp16 product, float transform and scale,
// one fp16 rounding.  suh null: plain copy of an already rotated input.
__device__ __forceinline__ void rotate_block(const __half* __restrict__ src, const __half* __restrict__ suh, int lane,
                                             __half (&h)[4])
{
    float v[4];
    if (suh) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float xv = __half2float(src[lane + 32 * i]);
            v[i] = __half2float(__float2half_rn(__fmul_rn(xv, __half2float(suh[lane + 32 * i]))));
        }
        warp_fwht128(v, lane);
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __float2half_rn(__fmul_rn(v[i], kHadScale));
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = src[lane + 32 * i];
    }
}

// ---------------------------------------------------------------------------
// tensor-core MMA (m16n8k16, fp16 inputs, fp32 accumulate)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(const uint32_t (&a)[4], uint32_t b0, uint32_t b1, float (&d)[4])
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Output element store in the requested dtype (0 = fp16, 1 = bf16, 2 = fp32).
__device__ __forceinline__ void store_out(void* out, size_t idx, float v, int dtype)
{
    if (dtype == 0) reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v);
    else if (dtype == 1) reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
    else reinterpret_cast<float*>(out)[idx] = v;
}

}  // namespace exl3b200
