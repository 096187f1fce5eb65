/*
 * dispatch/dispatch.h (portable subset) -- TEST INFRASTRUCTURE for the oracle build.
 *
 * The reference fans work out with Apple libdispatch:
 *   dispatch_apply_f(n, dispatch_get_global_queue(QOS_CLASS_USER_INITIATED, 0), ctx, fn)
 * runs fn(ctx, i) for i in [0, n) on a thread pool and returns when all are done
 * (e.g. kernel/attention.c:201, :378, :540 and kernel/kv_cache.c:101).
 * Here the same contract is met with an OpenMP parallel loop (dynamic schedule,
 * one index per chunk, like GCD's work stealing).  The thread count follows
 * OMP_NUM_THREADS.  Only the oracle build includes this header.
 */
#ifndef ORACLE_COMPAT_DISPATCH_H
#define ORACLE_COMPAT_DISPATCH_H

#include <stddef.h>

typedef void *dispatch_queue_t;

#define QOS_CLASS_USER_INITIATED 0x19

static inline dispatch_queue_t dispatch_get_global_queue(long identifier, unsigned long flags)
{
    (void)identifier;
    (void)flags;
    return (dispatch_queue_t)0;
}

static inline void dispatch_apply_f(size_t iterations, dispatch_queue_t queue, void *context,
                                    void (*work)(void *, size_t))
{
    (void)queue;
    long n = (long)iterations;
#pragma omp parallel for schedule(dynamic, 1)
    for (long i = 0; i < n; i++) work(context, (size_t)i);
}

#endif /* ORACLE_COMPAT_DISPATCH_H */
