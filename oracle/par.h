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
#include <stdlib.h>
#include <unistd.h>

typedef void (*wo_piece_fn)(int piece, void *arg);

typedef struct {
    wo_piece_fn fn;
    void *arg;
    int pieces, workers, id;
} wo_worker;

static void *wo_worker_main(void *p) {
    wo_worker *w = p;
    for (int piece = w->id; piece < w->pieces; piece += w->workers) w->fn(piece, w->arg);
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
    pthread_t *tid = malloc((size_t)threads * sizeof *tid);
    wo_worker *ws = malloc((size_t)threads * sizeof *ws);
    for (int t = 0; t < threads; t++) {
        ws[t] = (wo_worker){fn, arg, pieces, threads, t};
        if (t > 0) pthread_create(&tid[t], NULL, wo_worker_main, &ws[t]);
    }
    wo_worker_main(&ws[0]);
    for (int t = 1; t < threads; t++) pthread_join(tid[t], NULL);
    free(ws);
    free(tid);
}

static inline int wo_cpu_count(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

#endif
