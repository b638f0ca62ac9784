/* Host check of csrc/ddmath.h (built and run by tests/test_abi.py): counts how often the
 * correctly rounded exp/log and the gate mapping built on them differ from the C library,
 * and prints the first disagreements so the test can decide which side is right. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "ddmath.h"

static uint64_t s = 0x9E3779B97F4A7C15ull;
static double u01(void) {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return (double)(s >> 11) * 0x1.0p-53;
}

int main(int argc, char **argv) {
    long n = argc > 1 ? atol(argv[1]) : 100000;
    long bad_e = 0, bad_l = 0, bad_g = 0;
    for (long i = 0; i < n; i++) {
        double x = (u01() * 2 - 1) * 40;
        double a = vx_exp(x), b = exp(x);
        if (memcmp(&a, &b, 8)) { if (bad_e++ < 8) printf("exp %a %a %a\n", x, a, b); }
        double y = 1.0 + exp((u01() * 2 - 1) * 20);
        double c = vx_log(y), d = log(y);
        if (memcmp(&c, &d, 8)) { if (bad_l++ < 8) printf("log %a %a %a\n", y, c, d); }
        double ga = (u01() * 2 - 1) * 30, al = (u01() * 2 - 1) * 3, gb = (u01() * 2 - 1) * 30,
               dt = (u01() * 2 - 1) * 3, be, gg;
        vx_gate_params(ga, al, gb, dt, &be, &gg);
        double bo = 1.0 / (1.0 + exp(-gb)), xx = ga + dt;
        double sp = xx > 20.0 ? xx : (xx < -20.0 ? exp(xx) : log(1.0 + exp(xx)));
        double go = -exp(al) * sp;
        if (memcmp(&be, &bo, 8) || memcmp(&gg, &go, 8)) bad_g++;
    }
    printf("n=%ld exp_mismatch=%ld log_mismatch=%ld gate_mismatch=%ld\n", n, bad_e, bad_l, bad_g);
    return 0;
}
