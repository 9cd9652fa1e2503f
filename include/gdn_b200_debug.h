/*
 * gdn_b200_debug.h -- entry points that only the index-checked debug build
 * (libgdn_b200_debug.so, compiled with -DGDN_DEBUG_CHECKS) exports.  They
 * exist to test the library's own failure handling; the regular
 * libgdn_b200.so does not export them.  No counterpart in the reference.
 */
#ifndef GDN_B200_DEBUG_H_
#define GDN_B200_DEBUG_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Makes one bounded device wait run out, on purpose and safely.  With the
 * wait budget lowered to `limit_cycles` SM cycles (1 <= limit_cycles <=
 * 2^33), one CTA of 128 threads allocates TMEM as the prefill kernels do,
 * initialises an mbarrier that nothing ever arrives on (no TMA, bulk copy or
 * MMA is in flight), and waits on it with the same bounded wait the prefill
 * and backward kernels use.  The wait gives up, records device status 2
 * (read and cleared by gdn_b200_read_device_status), and the CTA frees its
 * TMEM and returns; the budget is then restored to 2^33 cycles.
 * result[4] (host memory) receives: [0] 1 if the wait reported success (it
 * must not), [1] the CTA's "gave up" flag, [2] 1 once the CTA has freed its
 * TMEM and reached the end, [3] the number of threads whose wait gave up.
 * Synchronises `stream`.
 */
int gdn_b200_debug_wait_timeout_probe(int64_t limit_cycles, int *result, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_DEBUG_H_ */
