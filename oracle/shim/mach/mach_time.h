/* Stand-in for <mach/mach_time.h>, used only to compile the reference's CPU
 * sources as a test oracle.  Time base 1/1 over CLOCK_MONOTONIC ns.
 * Test infrastructure; never part of the product. */
#pragma once
#include <stdint.h>
#include <time.h>

typedef struct { uint32_t numer; uint32_t denom; } mach_timebase_info_data_t;

static inline int mach_timebase_info(mach_timebase_info_data_t* t) { t->numer = 1; t->denom = 1; return 0; }
static inline uint64_t mach_absolute_time(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}
