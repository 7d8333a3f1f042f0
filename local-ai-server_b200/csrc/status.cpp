// status.cpp - status strings and version of liblai_kernels.so.
#include "../../include/lai_kernels.h"

extern "C" {

const char *lai_status_string(int status) {
    switch (status) {
        case LAI_OK: return "ok";
        case LAI_ERR_INVALID: return "invalid argument";
        case LAI_ERR_CUDA: return "CUDA error";
        case LAI_ERR_RANGE: return "index out of range";
        case LAI_ERR_ALIAS: return "unsupported overlap of output and input";
        case LAI_ERR_NOMEM: return "out of device memory";
        case LAI_ERR_TOOBIG: return "size beyond the stated maximum";
        default: return "unknown status";
    }
}

int lai_version(void) { return 100; /* 0.1.0 */ }

}  // extern "C"
