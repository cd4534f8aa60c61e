// Version and status names of the neutrongt_b200 C ABI.
#include "common.cuh"

extern "C" int ngt_abi_version(void) { return 1; }

extern "C" const char *ngt_status_string(int status) {
    switch (status) {
        case NGT_OK: return "NGT_OK";
        case NGT_ERR_INVALID_ARGUMENT: return "NGT_ERR_INVALID_ARGUMENT";
        case NGT_ERR_UNSUPPORTED: return "NGT_ERR_UNSUPPORTED";
        case NGT_ERR_WORKSPACE: return "NGT_ERR_WORKSPACE";
        case NGT_ERR_CUDA: return "NGT_ERR_CUDA";
        case NGT_ERR_MISALIGNED: return "NGT_ERR_MISALIGNED";
        case NGT_ERR_TOO_LARGE: return "NGT_ERR_TOO_LARGE";
        default: return "NGT_ERR_UNKNOWN";
    }
}
