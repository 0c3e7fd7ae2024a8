// Library-level C-ABI entry points: version and status strings, the limit of the
// bounded device-side waits.
#include <atomic>

#include "exl3_capi_internal.h"

namespace exl3b200 {
// 0 = each kernel's own default (tensor-core pipeline 1 s, decode peer exchange 2 s)
static std::atomic<unsigned long long> g_wait_limit_ns{0};

unsigned long long wait_limit_ns(unsigned long long dflt)
{
    const unsigned long long v = g_wait_limit_ns.load(std::memory_order_relaxed);
    return v ? v : dflt;
}
}  // namespace exl3b200

extern "C" int exl3b200_set_wait_limit(unsigned long long ns)
{
    exl3b200::g_wait_limit_ns.store(ns, std::memory_order_relaxed);
    return EXL3B200_OK;
}

extern "C" int exl3b200_abi_version(void) { return EXL3B200_ABI_VERSION; }

extern "C" const char* exl3b200_status_string(int status)
{
    switch (status) {
        case EXL3B200_OK: return "ok";
        case EXL3B200_EBADSHAPE: return "bad shape";
        case EXL3B200_EBADBITS: return "unsupported bits per weight (K)";
        case EXL3B200_EBADCODEBOOK: return "unsupported codebook";
        case EXL3B200_EUNALIGNED: return "misaligned pointer or stride";
        case EXL3B200_ELAUNCH: return "kernel launch failed";
        case EXL3B200_EWORKSPACE: return "workspace too small";
        case EXL3B200_ENULL: return "null pointer";
        case EXL3B200_EBADARG: return "bad argument";
        case EXL3B200_ETIMEOUT: return "device wait timed out";
        case EXL3B200_EIO: return "file read failed (short read)";
        default: return "unknown status";
    }
}
