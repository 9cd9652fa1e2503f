// gdn_b200.cu -- single translation unit of libgdn_b200.so.  The kernels share
// one per-device status word (g_device_status), so the library is compiled
// as one unit rather than with relocatable device code.
#include "gdn_decode.cu"
#include "gdn_prefill.cu"
#include "gdn_prefill_bwd.cu"
#include "gdn_capi.cu"
#include "gdn_prefill_noalloc.cu"
#include "gdn_debug_probe.cu"  // compiled only with -DGDN_DEBUG_CHECKS
