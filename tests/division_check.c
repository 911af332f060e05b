/* Exhaustive check of the division used by the sensitivity kernel
 * (memboost_b200/csrc/quantize.cu, stats_kernel):
 *     r = RN(1/h),  q0 = RN(x * r),  q1 = RN(fma(RN(fma(-q0, h, x)), r, q0))
 * must equal RN(x / h) for every dividend x = w*w of an fp16 w and every fp32
 * divisor h.  Correct rounding depends only on the significands when nothing
 * overflows or underflows, so h runs over all 2^23 significands in [1, 2)
 * and x over every significand a square of an fp16 value can have (normal
 * and subnormal w), placed in [1, 2) and [2, 4).  Prints the mismatch count;
 * exit status 1 if any.  Used by tests/test_division.py. */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float X[4096];
static int NX;
static long long bad[256];
static int NT;

static void* work(void* arg) {
  long t = (long)arg;
  long long b = 0;
  for (uint32_t m = (uint32_t)t; m < (1u << 23); m += (uint32_t)NT) {
    uint32_t hb = 0x3F800000u | m;
    float h;
    memcpy(&h, &hb, 4);
    const float r = 1.0f / h;
    for (int i = 0; i < NX; ++i) {
      const float x = X[i];
      const float q0 = x * r;
      const float rem = fmaf(-q0, h, x);
      const float q1 = fmaf(rem, r, q0);
      if (q1 != x / h) ++b;
    }
  }
  bad[t] = b;
  return NULL;
}

int main(int argc, char** argv) {
  NT = argc > 1 ? atoi(argv[1]) : 8;
  if (NT < 1) NT = 1;
  if (NT > 256) NT = 256;
  for (int m = 0; m < 1024; ++m) {
    const double s = (1024.0 + m) / 1024.0;
    X[NX++] = (float)(s * s);
  }
  for (int m = 1; m < 1024; ++m) {
    int e;
    const double f = frexp((double)m * m, &e);
    X[NX++] = (float)(f * 2.0);
    X[NX++] = (float)(f * 4.0);
  }
  pthread_t th[256];
  for (long t = 0; t < NT; ++t) pthread_create(&th[t], NULL, work, (void*)t);
  long long tot = 0;
  for (int t = 0; t < NT; ++t) {
    pthread_join(th[t], NULL);
    tot += bad[t];
  }
  printf("dividends %d, divisor significands %u, mismatches %lld\n", NX, 1u << 23, tot);
  return tot != 0;
}
