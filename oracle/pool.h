/* pool.h -- a tiny task pool for the oracle (TEST INFRASTRUCTURE ONLY).
 * oracle_parallel_for(tasks, threads, f, ctx) calls f(ctx, i) once for every i < tasks, as
 * Pool::run does (src/threads.rs:103-145). Each task owns its outputs, so results do not depend
 * on the thread count. */
#ifndef TELMO_ORACLE_POOL_H
#define TELMO_ORACLE_POOL_H
#include <stddef.h>
void oracle_parallel_for(size_t tasks, int threads, void (*f)(void *, size_t), void *ctx);
#endif
