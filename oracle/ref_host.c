/* Test infrastructure (parity oracle / CPU baseline), not product code.
 *
 * Host services that the reference's kernels.c imports from its WebAssembly embedder, for the native build of
 * that file under oracle/_ref/:
 *   - js_now(): the profiler clock imported as env.now (kernels.c:20, cpu-worker.js:14), in milliseconds;
 *   - memory.atomic.wait32 / notify used by the MT barrier and worker park loop (kernels.c:46-58, 441-449),
 *     as Linux futexes;
 *   - h2shim_start_helpers(): starts threads 1..nth-1 parked in worker_loop(tid), as the leader worker does with
 *     Web Workers (cpu-worker.js:141-149).
 */
#define _GNU_SOURCE
#include <limits.h>
#include <linux/futex.h>
#include <pthread.h>
#include <stdint.h>
#include <sys/syscall.h>
#include <time.h>
#include <unistd.h>

double js_now(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec * 1e3 + (double)ts.tv_nsec * 1e-6;
}

int h2shim_wait32(int* addr, int expected, long long timeout_ns) {
  if (__atomic_load_n(addr, __ATOMIC_SEQ_CST) != expected) return 1; /* "not-equal" */
  struct timespec ts, *tp = 0;
  if (timeout_ns >= 0) {
    ts.tv_sec = (time_t)(timeout_ns / 1000000000LL);
    ts.tv_nsec = (long)(timeout_ns % 1000000000LL);
    tp = &ts;
  }
  long r = syscall(SYS_futex, addr, FUTEX_WAIT_PRIVATE, expected, tp, 0, 0);
  return r == 0 ? 0 : 2; /* "ok" or "timed-out"/interrupted */
}

int h2shim_notify(int* addr, int count) {
  long r = syscall(SYS_futex, addr, FUTEX_WAKE_PRIVATE, count < 0 ? INT_MAX : count, 0, 0, 0);
  return (int)r;
}

#ifdef MT
extern void worker_loop(int tid);
static int helpers_started;

static void* helper_main(void* arg) {
  worker_loop((int)(intptr_t)arg); /* never returns */
  return 0;
}

/* Start helper threads 1..nth-1 once per process; later calls may only ask for as many as already exist. */
int h2shim_start_helpers(int nth) {
  if (helpers_started) return nth <= helpers_started ? 0 : -1;
  for (int t = 1; t < nth; t++) {
    pthread_t th;
    pthread_attr_t at;
    pthread_attr_init(&at);
    pthread_attr_setdetachstate(&at, PTHREAD_CREATE_DETACHED);
    if (pthread_create(&th, &at, helper_main, (void*)(intptr_t)t) != 0) return -2;
    pthread_attr_destroy(&at);
  }
  helpers_started = nth;
  return 0;
}
#else
int h2shim_start_helpers(int nth) { return nth <= 1 ? 0 : -1; }
#endif
