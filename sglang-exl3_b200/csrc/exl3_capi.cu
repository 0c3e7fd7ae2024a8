// Library-level C-ABI entry points: version and status strings.
#include "exl3_capi_internal.h"

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
