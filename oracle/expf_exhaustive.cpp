// ORACLE support — test infrastructure only.
//
// Exhaustive check of q3o_cr_expf: for every binary32 pattern in [lo, hi]
// (default: every float in [-104, -0], the domain of exp(x - max) in the
// sampler) compare against expl rounded to binary32, and count where glibc
// expf differs from the correctly rounded value.
//   usage: expf_exhaustive [lo_bits_hex hi_bits_hex [threads]]
// Prints one line: "checked=N cr_mismatch=A libm_mismatch=B".

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "q3s_oracle.h"

namespace {

struct Job {
  uint64_t lo, hi;
  uint64_t checked, cr_bad, libm_bad;
};

inline float bits_to_f(uint32_t b) {
  float f;
  memcpy(&f, &b, 4);
  return f;
}

inline uint32_t f_to_bits(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

void* work(void* arg) {
  Job* j = (Job*)arg;
  for (uint64_t b = j->lo; b <= j->hi; ++b) {
    float x = bits_to_f((uint32_t)b);
    float ref = (float)expl((long double)x);
    float cr = q3o_cr_expf(x);
    float lm = expf(x);
    j->checked++;
    if (f_to_bits(cr) != f_to_bits(ref)) {
      if (j->cr_bad < 8) fprintf(stderr, "cr mismatch x=%a cr=%a ref=%a\n", x, cr, ref);
      j->cr_bad++;
    }
    if (f_to_bits(lm) != f_to_bits(ref)) j->libm_bad++;
  }
  return nullptr;
}

}  // namespace

int main(int argc, char** argv) {
  uint64_t lo = 0x80000000u, hi = 0xC2D00000u;  // -0 .. -104
  int threads = 8;
  if (argc >= 3) {
    lo = strtoull(argv[1], nullptr, 16);
    hi = strtoull(argv[2], nullptr, 16);
  }
  if (argc >= 4) threads = atoi(argv[3]);
  if (threads < 1) threads = 1;
  std::vector<Job> jobs(threads);
  std::vector<pthread_t> tids(threads);
  uint64_t span = hi - lo + 1;
  for (int t = 0; t < threads; ++t) {
    jobs[t].lo = lo + span * t / threads;
    jobs[t].hi = lo + span * (t + 1) / threads - 1;
    jobs[t].checked = jobs[t].cr_bad = jobs[t].libm_bad = 0;
    pthread_create(&tids[t], nullptr, work, &jobs[t]);
  }
  uint64_t checked = 0, cr_bad = 0, libm_bad = 0;
  for (int t = 0; t < threads; ++t) {
    pthread_join(tids[t], nullptr);
    checked += jobs[t].checked;
    cr_bad += jobs[t].cr_bad;
    libm_bad += jobs[t].libm_bad;
  }
  printf("checked=%llu cr_mismatch=%llu libm_mismatch=%llu\n", (unsigned long long)checked,
         (unsigned long long)cr_bad, (unsigned long long)libm_bad);
  return cr_bad == 0 ? 0 : 1;
}
