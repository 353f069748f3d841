// gdn_abi.cu — version and status-text entry points of the C ABI.
#include "../../include/gdn_b200.h"

extern "C" int gdn_abi_version(void) { return 4; }

extern "C" const char* gdn_strerror(int status) {
    switch (status) {
        case GDN_OK: return "ok";
        case GDN_ERR_INVALID: return "invalid argument (null pointer, negative size or bad flag)";
        case GDN_ERR_UNSUPPORTED: return "unsupported shape (needs K == V == 128 and HV % H == 0)";
        case GDN_ERR_ALIGN: return "misaligned pointer (see the alignment rules in gdn_b200.h)";
        case GDN_ERR_CUDA: return "CUDA launch failed";
        case GDN_ERR_DEVICE: return "a kernel reported a device-side error (bounded wait timed out)";
        case GDN_ERR_TOO_LARGE: return "problem needs more than the 16 MiB scratch of gdn_prefill_fwd_noalloc";
        default: return "unknown status";
    }
}
