/* Host check of the blend's quotient routine (divide_by in
 * vocal-fast-rs_b200/csrc/exact_common.cuh): the same IEEE double operations
 * (one multiply, four fused multiply-adds, y = RN(1/S)) against the correctly
 * rounded quotient t / S, on random and near-midpoint cases in the fast
 * path's domain (S in [2^-500, 2^500], |t| in [2^-400, 2^400]).  IEEE-754
 * multiply and fma are correctly rounded on the CPU and the GPU alike, so a
 * mismatch here is a mismatch there.  Prints "cases mismatches" and exits 1
 * on any mismatch.  Built by tests/test_division.py with -ffp-contract=off.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static uint64_t rng = 0x9E3779B97F4A7C15ull;
static uint64_t next_u64(void) {
    rng ^= rng << 13;
    rng ^= rng >> 7;
    rng ^= rng << 17;
    return rng;
}
static double uniform(void) { return (double)(next_u64() >> 11) * 0x1p-53; }

/* the fast path of divide_by */
static double markstein(double t, double s, double y) {
    const double q0 = t * y;
    const double r0 = fma(-s, q0, t);
    const double q1 = fma(r0, y, q0);
    const double r1 = fma(-s, q1, t);
    return fma(r1, y, q1);
}

static int same(double a, double b) { return memcmp(&a, &b, sizeof a) == 0; }

static double random_double(int emin, int emax) {
    const int e = emin + (int)(next_u64() % (uint64_t)(emax - emin + 1));
    double m = 1.0 + uniform();
    if (next_u64() & 1) m = -m;
    return ldexp(m, e);
}

int main(int argc, char **argv) {
    const long n = argc > 1 ? atol(argv[1]) : 4000000;
    long bad = 0, cases = 0;
    for (long i = 0; i < n; ++i) {
        double t, s;
        switch (i & 3) {
            case 0: { /* the blend's shape: an f32 value times a weight, S a sum of weights */
                const float v = (float)((uniform() - 0.5) * 8.0);
                int count = 1 + (int)(next_u64() % 8);
                double w[8], sum = -0.0;
                for (int k = 0; k < count; ++k) {
                    const float d = (float)(ldexp(0.5 + uniform(), (int)(next_u64() % 40) - 10));
                    const double sd = (double)(d > 1e-12f ? d : 1e-12f);
                    w[k] = 1.0 / (sd * sd);
                    sum = sum + w[k];
                }
                t = (double)v * w[next_u64() % count];
                s = sum;
                break;
            }
            case 1: /* arbitrary significands across the domain */
                t = random_double(-400, 400);
                s = fabs(random_double(-400, 400));
                break;
            case 2: { /* quotients next to a rounding midpoint */
                s = fabs(random_double(-60, 60));
                const double q = fabs(random_double(-60, 60));
                const double mid = q + 0.5 * (nextafter(q, INFINITY) - q);
                t = s * mid; /* rounded: t / s lands within a few ulps of the midpoint */
                if (next_u64() & 1) t = nextafter(t, (next_u64() & 1) ? INFINITY : -INFINITY);
                break;
            }
            default: /* small-integer ratios and powers of two */
                s = ldexp((double)(1 + next_u64() % 4096), (int)(next_u64() % 64) - 32);
                t = ldexp((double)(1 + next_u64() % 4096), (int)(next_u64() % 64) - 32);
                break;
        }
        if (!(fabs(s) >= 0x1p-500 && fabs(s) <= 0x1p500) || !(fabs(t) >= 0x1p-400 && fabs(t) <= 0x1p400)) continue;
        ++cases;
        const double y = 1.0 / s;
        const double want = t / s, got = markstein(t, s, y);
        if (!same(want, got)) {
            if (bad < 5) fprintf(stderr, "t=%a s=%a want=%a got=%a\n", t, s, want, got);
            ++bad;
        }
    }
    printf("%ld %ld\n", cases, bad);
    return bad != 0;
}
