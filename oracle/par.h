/*
 * par.h — a static parallel-for on POSIX threads for the CPU oracle's timed
 * baseline (test infrastructure). It stands in for algo-tensor's
 * tensor.Parallel (lut.go:110, :191): pieces are fixed before any thread
 * starts, and every piece writes disjoint outputs, so results do not depend
 * on the thread count. No OpenMP: the process also hosts torch's own runtime.
 */
#ifndef WHISTLE_ORACLE_PAR_H
#define WHISTLE_ORACLE_PAR_H

#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <unistd.h>

typedef void (*wo_piece_fn)(int piece, void *arg);

static inline int wo_cpu_count(void);

/* A persistent pool (created on first use), standing in for the cheap
 * goroutines behind tensor.Parallel: a job costs a wake-up, not a thread
 * start. Idle workers spin for a while on the job counter before they sleep,
 * so back-to-back calls (the timed baseline) hand work over in about a
 * microsecond. Worker k runs pieces k, k + n, ... of each job with n
 * threads; the caller runs the pieces of thread 0 and waits for the rest.
 * One job at a time. */
typedef struct {
    pthread_mutex_t mu;
    pthread_cond_t go;
    wo_piece_fn fn;
    void *arg;
    int pieces, threads, size;
    atomic_int gen, left;
} wo_pool_t;

static wo_pool_t wo_pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, NULL, NULL, 0, 0, 0, 0, 0};
static pthread_mutex_t wo_pool_call = PTHREAD_MUTEX_INITIALIZER;

static inline void wo_relax(void) {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#endif
}

static void *wo_pool_main(void *p) {
    const int id = (int)(intptr_t)p;
    int seen = 0;
    for (;;) {
        int g = atomic_load_explicit(&wo_pool.gen, memory_order_acquire);
        for (int spin = 0; g == seen && spin < (1 << 16); spin++) {
            wo_relax();
            g = atomic_load_explicit(&wo_pool.gen, memory_order_acquire);
        }
        if (g == seen) {
            pthread_mutex_lock(&wo_pool.mu);
            while ((g = atomic_load_explicit(&wo_pool.gen, memory_order_acquire)) == seen)
                pthread_cond_wait(&wo_pool.go, &wo_pool.mu);
            pthread_mutex_unlock(&wo_pool.mu);
        }
        seen = g;
        const int threads = wo_pool.threads;
        if (id < threads) {
            for (int piece = id; piece < wo_pool.pieces; piece += threads) wo_pool.fn(piece, wo_pool.arg);
            atomic_fetch_sub_explicit(&wo_pool.left, 1, memory_order_release);
        }
    }
    return NULL;
}

/* Runs fn(piece, arg) for piece in [0, pieces) on up to `threads` threads,
 * piece i on thread i mod threads. */
static inline void wo_parallel_for(int pieces, int threads, wo_piece_fn fn, void *arg) {
    if (threads > pieces) threads = pieces;
    if (threads <= 1) {
        for (int i = 0; i < pieces; i++) fn(i, arg);
        return;
    }
    pthread_mutex_lock(&wo_pool_call);
    if (wo_pool.size == 0) {
        const int n = wo_cpu_count();
        for (int k = 1; k < n; k++) {
            pthread_t t;
            if (pthread_create(&t, NULL, wo_pool_main, (void *)(intptr_t)k) != 0) break;
            pthread_detach(t);
            wo_pool.size = k;
        }
    }
    if (threads > wo_pool.size + 1) threads = wo_pool.size + 1;
    if (threads <= 1) {
        pthread_mutex_unlock(&wo_pool_call);
        for (int i = 0; i < pieces; i++) fn(i, arg);
        return;
    }
    wo_pool.fn = fn;
    wo_pool.arg = arg;
    wo_pool.pieces = pieces;
    wo_pool.threads = threads;
    atomic_store_explicit(&wo_pool.left, threads - 1, memory_order_relaxed);
    pthread_mutex_lock(&wo_pool.mu);
    atomic_fetch_add_explicit(&wo_pool.gen, 1, memory_order_release);
    pthread_cond_broadcast(&wo_pool.go);
    pthread_mutex_unlock(&wo_pool.mu);
    for (int piece = 0; piece < pieces; piece += threads) fn(piece, arg);
    while (atomic_load_explicit(&wo_pool.left, memory_order_acquire) > 0) wo_relax();
    pthread_mutex_unlock(&wo_pool_call);
}

static inline int wo_cpu_count(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

#endif
