/*
 * POSIX thread pool with the same four entry points as the reference's Win32 pool
 * (src/threadpool.h:8-13 in DavidPandleton/vx27), so the reference's own caller code
 * (src/vx27_block.c) links against it unchanged. TEST / BASELINE INFRASTRUCTURE ONLY.
 */
#ifndef QL_THREADPOOL_H
#define QL_THREADPOOL_H
#include <stddef.h>

typedef struct threadpool threadpool;

threadpool *tp_create(int n_threads, char *err, size_t errlen);
void tp_free(threadpool *tp);
int tp_threads(const threadpool *tp);
/* Runs fn(arg, tid, nthreads) on every worker and returns when all have finished. */
int tp_run(threadpool *tp, void (*fn)(void *, int, int), void *arg);

#endif
