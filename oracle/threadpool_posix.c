/*
 * POSIX implementation of the reference thread-pool interface (src/threadpool.h:8-13).
 * The reference pool (src/threadpool.c:99-203) is Win32-only (CreateThread,
 * SleepConditionVariableCS); this one uses pthreads. Worker 0 is the calling thread,
 * as in the reference (tp_run runs fn(arg, 0, n) on the caller). A generation counter
 * releases the workers; a countdown under the same mutex signals completion.
 * TEST / BASELINE INFRASTRUCTURE ONLY.
 */
#define _POSIX_C_SOURCE 200809L
#include "threadpool.h"
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>

struct threadpool {
    int n;
    pthread_t *th;
    pthread_mutex_t mu;
    pthread_cond_t go, done;
    unsigned long gen;
    int pending, quit;
    void (*fn)(void *, int, int);
    void *arg;
};

typedef struct { threadpool *tp; int tid; } tp_worker_arg;

static void *tp_worker(void *p) {
    tp_worker_arg *wa = (tp_worker_arg *)p;
    threadpool *tp = wa->tp;
    int tid = wa->tid;
    free(wa);
    unsigned long seen = 0;
    for (;;) {
        pthread_mutex_lock(&tp->mu);
        while (tp->gen == seen && !tp->quit) pthread_cond_wait(&tp->go, &tp->mu);
        if (tp->quit) { pthread_mutex_unlock(&tp->mu); return NULL; }
        seen = tp->gen;
        void (*fn)(void *, int, int) = tp->fn;
        void *arg = tp->arg;
        pthread_mutex_unlock(&tp->mu);
        fn(arg, tid, tp->n);
        pthread_mutex_lock(&tp->mu);
        if (--tp->pending == 0) pthread_cond_signal(&tp->done);
        pthread_mutex_unlock(&tp->mu);
    }
}

threadpool *tp_create(int n_threads, char *err, size_t errlen) {
    if (n_threads < 1) n_threads = 1;
    threadpool *tp = (threadpool *)calloc(1, sizeof *tp);
    if (!tp) { if (err) snprintf(err, errlen, "tp_create: out of memory"); return NULL; }
    tp->n = n_threads;
    pthread_mutex_init(&tp->mu, NULL);
    pthread_cond_init(&tp->go, NULL);
    pthread_cond_init(&tp->done, NULL);
    tp->th = (pthread_t *)calloc((size_t)n_threads, sizeof(pthread_t));
    for (int t = 1; t < n_threads; t++) {
        tp_worker_arg *wa = (tp_worker_arg *)malloc(sizeof *wa);
        wa->tp = tp; wa->tid = t;
        if (pthread_create(&tp->th[t], NULL, tp_worker, wa) != 0) {
            if (err) snprintf(err, errlen, "tp_create: pthread_create failed at %d", t);
            free(wa);
            tp->n = t;
            tp_free(tp);
            return NULL;
        }
    }
    return tp;
}

int tp_threads(const threadpool *tp) { return tp ? tp->n : 1; }

int tp_run(threadpool *tp, void (*fn)(void *, int, int), void *arg) {
    if (!tp || tp->n == 1) { fn(arg, 0, 1); return 0; }
    pthread_mutex_lock(&tp->mu);
    tp->fn = fn; tp->arg = arg;
    tp->pending = tp->n - 1;
    tp->gen++;
    pthread_cond_broadcast(&tp->go);
    pthread_mutex_unlock(&tp->mu);
    fn(arg, 0, tp->n);
    pthread_mutex_lock(&tp->mu);
    while (tp->pending > 0) pthread_cond_wait(&tp->done, &tp->mu);
    pthread_mutex_unlock(&tp->mu);
    return 0;
}

void tp_free(threadpool *tp) {
    if (!tp) return;
    pthread_mutex_lock(&tp->mu);
    tp->quit = 1;
    pthread_cond_broadcast(&tp->go);
    pthread_mutex_unlock(&tp->mu);
    for (int t = 1; t < tp->n; t++) pthread_join(tp->th[t], NULL);
    pthread_mutex_destroy(&tp->mu);
    pthread_cond_destroy(&tp->go);
    pthread_cond_destroy(&tp->done);
    free(tp->th);
    free(tp);
}
