// Checkpoint reader: byte ranges of an open file (a safetensors shard) copied
// straight into device memory, or into host memory.
//
// B200 boxes keep HBM behind PCIe, so a tensor's bytes have to cross from the file
// into a pinned host buffer and then over DMA into HBM.  The caller hands over one
// pinned staging buffer; it is split into one slot per reader thread.  Each thread
// takes the next chunk of the range list, waits until the DMA that last used its
// slot has finished, pread()s the chunk into the slot and enqueues the slot's
// host-to-device copy on the caller's stream.  Disk reads of one thread therefore
// overlap the copies of the others, and no byte passes through pageable memory.
// Host destinations are read into directly, without staging or any CUDA call.
#include "exl3_capi_internal.h"

#include <atomic>
#include <cerrno>
#include <fcntl.h>
#include <thread>
#include <unistd.h>
#include <vector>

namespace {

constexpr long long kHostChunk = 16ll << 20;  // host destinations: parallel grain
constexpr size_t kSlotAlign = 4096;
constexpr int kMaxThreads = 64;

struct Chunk {
    long long off, size;
    char* dst;
};

bool pread_full(int fd, char* buf, long long n, long long off)
{
    while (n > 0) {
        const ssize_t r = pread(fd, buf, (size_t) std::min(n, 1ll << 30), (off_t) off);
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return false;  // error or end of file before the range ends
        buf += r;
        off += r;
        n -= r;
    }
    return true;
}

void drop_pages(int fd, long long off, long long n)
{
#ifdef POSIX_FADV_DONTNEED
    posix_fadvise(fd, (off_t) off, (off_t) n, POSIX_FADV_DONTNEED);
#else
    (void) fd, (void) off, (void) n;
#endif
}

}  // namespace

extern "C" int exl3b200_read_ranges(int fd, const long long* offsets, const long long* sizes, void* const* dst,
                                    int count, int dst_on_device, void* staging, size_t staging_bytes, int threads,
                                    int drop_cache, void* stream)
{
    if (fd < 0 || count < 0 || threads < 1 || threads > kMaxThreads) return EXL3B200_EBADARG;
    if (count == 0) return EXL3B200_OK;
    if (!offsets || !sizes || !dst) return EXL3B200_ENULL;
    for (int i = 0; i < count; ++i) {
        if (offsets[i] < 0 || sizes[i] < 0) return EXL3B200_EBADARG;
        if (sizes[i] > 0 && !dst[i]) return EXL3B200_ENULL;
    }
    long long grain = kHostChunk;
    if (dst_on_device) {
        if (!staging) return EXL3B200_ENULL;
        const size_t slot = (staging_bytes / (size_t) threads) & ~(kSlotAlign - 1);
        if (slot < kSlotAlign) return EXL3B200_EWORKSPACE;
        grain = (long long) slot;
    }

    std::vector<Chunk> chunks;
    for (int i = 0; i < count; ++i)
        for (long long done = 0; done < sizes[i]; done += grain)
            chunks.push_back({offsets[i] + done, std::min(grain, sizes[i] - done), (char*) dst[i] + done});
    if (chunks.empty()) return EXL3B200_OK;
    const int nthreads = (int) std::min<size_t>((size_t) threads, chunks.size());

    int device = 0;
    if (dst_on_device && cudaGetDevice(&device) != cudaSuccess) return EXL3B200_ELAUNCH;
    cudaStream_t st = (cudaStream_t) stream;
    std::atomic<size_t> next{0};
    std::atomic<int> status{EXL3B200_OK};
    auto fail = [&](int code) {
        int ok = EXL3B200_OK;
        status.compare_exchange_strong(ok, code);
    };

    auto worker = [&](int w) {
        cudaEvent_t done_ev = nullptr;
        bool pending = false;
        char* slot = dst_on_device ? (char*) staging + (size_t) w * (size_t) grain : nullptr;
        if (dst_on_device) {
            // the CUDA current device is per thread: follow the caller's
            if (cudaSetDevice(device) != cudaSuccess ||
                cudaEventCreateWithFlags(&done_ev, cudaEventDisableTiming) != cudaSuccess) {
                fail(EXL3B200_ELAUNCH);
                return;
            }
        }
        for (;;) {
            const size_t i = next.fetch_add(1);
            if (i >= chunks.size() || status.load() != EXL3B200_OK) break;
            const Chunk& c = chunks[i];
            if (!dst_on_device) {
                if (!pread_full(fd, c.dst, c.size, c.off)) fail(EXL3B200_EIO);
            } else {
                if (pending && cudaEventSynchronize(done_ev) != cudaSuccess) {
                    fail(EXL3B200_ELAUNCH);
                    break;
                }
                pending = false;
                if (!pread_full(fd, slot, c.size, c.off)) {
                    fail(EXL3B200_EIO);
                    break;
                }
                if (cudaMemcpyAsync(c.dst, slot, (size_t) c.size, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                    cudaEventRecord(done_ev, st) != cudaSuccess) {
                    fail(EXL3B200_ELAUNCH);
                    break;
                }
                pending = true;
            }
            if (drop_cache) drop_pages(fd, c.off, c.size);
        }
        if (done_ev) {
            // the slot must not be reused (or the staging buffer freed) under a copy
            if (pending && cudaEventSynchronize(done_ev) != cudaSuccess) fail(EXL3B200_ELAUNCH);
            cudaEventDestroy(done_ev);
        }
    };

    std::vector<std::thread> pool;
    pool.reserve((size_t) nthreads - 1);
    for (int w = 1; w < nthreads; ++w) pool.emplace_back(worker, w);
    worker(0);
    for (auto& t : pool) t.join();
    return status.load();
}
