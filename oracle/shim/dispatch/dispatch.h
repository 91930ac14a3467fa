/* Stand-in for libdispatch, used only to compile the reference's CPU sources
 * as a test oracle.  dispatch_apply runs the iterations in order on the
 * calling thread.  Test infrastructure; never part of the product. */
#pragma once
#include <stddef.h>

typedef void* dispatch_queue_t;
#define QOS_CLASS_USER_INTERACTIVE 0x21

static inline dispatch_queue_t dispatch_get_global_queue(long, unsigned long) { return nullptr; }

template <typename F>
static inline void dispatch_apply(size_t n, dispatch_queue_t, F&& f) {
    for (size_t i = 0; i < n; i++) f(i);
}
