// Test infrastructure: runs the reference's own device decode functions on a GPU
// and dumps their results, to pin the CPU oracle's round-to-nearest codebooks
// and trellis window extraction against the reference itself.
//
// Compiled by oracle/build_ref.py against the read-only reference tree
// (-I <reference>/csrc); the reference headers are used in place, not copied:
//   decode_3inst<cb>            csrc/quant/codebook.cuh:56-90
//   dq_dispatch<bits, cb>       csrc/quant/exl3_dq.cuh:259-293
// Output (argv[1], little-endian raw):
//   "EXL3CBD1"
//   for cb in 0..2: 65536 x uint16       codebook table
//   uint32 ntiles
//   for K in 1..8: ntiles*16K x uint16   input tiles (splitmix64, seed 0x5eed + K)
//                  for cb in 0..2: ntiles*256 x uint16 decoded values in t order
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <vector>
#include <cuda_runtime.h>
#include "util.cuh"
#include "ptx.cuh"
#include "quant/exl3_dq.cuh"

template <int cb>
__global__ void table_kernel(uint16_t* out)
{
    int w = blockIdx.x * blockDim.x + threadIdx.x;
    if (w < 65536) out[w] = __half_as_ushort(decode_3inst<cb>((uint32_t) w));
}

template <int bits, int cb>
__global__ void tile_kernel(const uint16_t* tiles, uint16_t* out)
{
    const int tile = blockIdx.x;
    const int lane = threadIdx.x;
    const uint32_t* ptr = reinterpret_cast<const uint32_t*>(tiles + (size_t) tile * 16 * bits);
    FragB f0, f1;
    dq_dispatch<bits, cb>(ptr, lane << 3, f0, f1);
    uint16_t* o = out + (size_t) tile * 256 + lane * 8;
    o[0] = __half_as_ushort(__low2half(f0[0]));
    o[1] = __half_as_ushort(__high2half(f0[0]));
    o[2] = __half_as_ushort(__low2half(f0[1]));
    o[3] = __half_as_ushort(__high2half(f0[1]));
    o[4] = __half_as_ushort(__low2half(f1[0]));
    o[5] = __half_as_ushort(__high2half(f1[0]));
    o[6] = __half_as_ushort(__low2half(f1[1]));
    o[7] = __half_as_ushort(__high2half(f1[1]));
}

static uint64_t splitmix64(uint64_t& s)
{
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

#define CK(x) do { cudaError_t e_ = (x); if (e_ != cudaSuccess) { \
    fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); return 1; } } while (0)

template <int bits, int cb>
static int run_tiles(const uint16_t* d_tiles, uint16_t* d_out, int ntiles)
{
    tile_kernel<bits, cb><<<ntiles, 32>>>(d_tiles, d_out);
    CK(cudaGetLastError());
    return 0;
}

template <int bits>
static int run_bits(FILE* f, int ntiles)
{
    const size_t nw = (size_t) ntiles * 16 * bits;
    std::vector<uint16_t> tiles(nw);
    uint64_t s = 0x5eedull + bits;
    for (size_t i = 0; i < nw; ++i) tiles[i] = (uint16_t) (splitmix64(s) & 0xffff);
    uint16_t *d_tiles = nullptr, *d_out = nullptr;
    CK(cudaMalloc(&d_tiles, nw * 2));
    CK(cudaMalloc(&d_out, (size_t) ntiles * 256 * 2));
    CK(cudaMemcpy(d_tiles, tiles.data(), nw * 2, cudaMemcpyHostToDevice));
    fwrite(tiles.data(), 2, nw, f);
    std::vector<uint16_t> out((size_t) ntiles * 256);
    for (int cb = 0; cb < 3; ++cb) {
        int rc = cb == 0 ? run_tiles<bits, 0>(d_tiles, d_out, ntiles)
               : cb == 1 ? run_tiles<bits, 1>(d_tiles, d_out, ntiles)
                         : run_tiles<bits, 2>(d_tiles, d_out, ntiles);
        if (rc) return rc;
        CK(cudaMemcpy(out.data(), d_out, out.size() * 2, cudaMemcpyDeviceToHost));
        fwrite(out.data(), 2, out.size(), f);
    }
    CK(cudaFree(d_tiles));
    CK(cudaFree(d_out));
    return 0;
}

int main(int argc, char** argv)
{
    if (argc < 2) { fprintf(stderr, "usage: %s OUT\n", argv[0]); return 2; }
    FILE* f = fopen(argv[1], "wb");
    if (!f) { perror("fopen"); return 2; }
    fwrite("EXL3CBD1", 1, 8, f);
    uint16_t* d_tab = nullptr;
    CK(cudaMalloc(&d_tab, 65536 * 2));
    std::vector<uint16_t> tab(65536);
    for (int cb = 0; cb < 3; ++cb) {
        if (cb == 0) table_kernel<0><<<256, 256>>>(d_tab);
        if (cb == 1) table_kernel<1><<<256, 256>>>(d_tab);
        if (cb == 2) table_kernel<2><<<256, 256>>>(d_tab);
        CK(cudaGetLastError());
        CK(cudaMemcpy(tab.data(), d_tab, 65536 * 2, cudaMemcpyDeviceToHost));
        fwrite(tab.data(), 2, 65536, f);
    }
    CK(cudaFree(d_tab));
    const uint32_t ntiles = 64;
    fwrite(&ntiles, 4, 1, f);
    int rc = run_bits<1>(f, ntiles) || run_bits<2>(f, ntiles) || run_bits<3>(f, ntiles) ||
             run_bits<4>(f, ntiles) || run_bits<5>(f, ntiles) || run_bits<6>(f, ntiles) ||
             run_bits<7>(f, ntiles) || run_bits<8>(f, ntiles);
    fclose(f);
    if (rc) return rc;
    printf("ok\n");
    return 0;
}
