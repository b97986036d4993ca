/* pool.c -- see pool.h. TEST INFRASTRUCTURE ONLY. */
#include "pool.h"

#include <pthread.h>
#include <stdlib.h>

typedef struct {
    size_t tasks;
    size_t next; /* guarded by lock */
    pthread_mutex_t lock;
    void (*f)(void *, size_t);
    void *ctx;
} pool_job;

static void *worker(void *arg)
{
    pool_job *J = (pool_job *)arg;
    for (;;) {
        pthread_mutex_lock(&J->lock);
        size_t t = J->next++;
        pthread_mutex_unlock(&J->lock);
        if (t >= J->tasks) break;
        J->f(J->ctx, t);
    }
    return NULL;
}

void oracle_parallel_for(size_t tasks, int threads, void (*f)(void *, size_t), void *ctx)
{
    if (tasks == 0) return;
    if (threads <= 1 || tasks == 1) {
        for (size_t t = 0; t < tasks; t++) f(ctx, t);
        return;
    }
    pool_job J;
    J.tasks = tasks;
    J.next = 0;
    J.f = f;
    J.ctx = ctx;
    pthread_mutex_init(&J.lock, NULL);
    int extra = threads - 1;
    if ((size_t)extra > tasks - 1) extra = (int)(tasks - 1);
    pthread_t *ids = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)extra);
    int started = 0;
    for (int i = 0; i < extra; i++)
        if (pthread_create(&ids[i], NULL, worker, &J) == 0) started++;
        else break;
    worker(&J);
    for (int i = 0; i < started; i++) pthread_join(ids[i], NULL);
    free(ids);
    pthread_mutex_destroy(&J.lock);
}
