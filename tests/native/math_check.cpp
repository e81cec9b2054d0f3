// Host check of gateddeltanet_b200/csrc/gdn_math.h against the host libm
// (test infrastructure, compiled by tests/test_math_cpu.py): counts the
// inputs on a sweep of all floats in [lo, hi] (every `stride`-th bit
// pattern) where gdn_expf / gdn_sigmoidf differ from expf / the reference
// sigmoid formula (c_impl/gdn_model.cpp:1307-1316).
#include "gdn_math.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

static float ref_sigmoid(float x) {
    if (x >= 0.0f) {
        float z = expf(-x);
        return 1.0f / (1.0f + z);
    }
    float z = expf(x);
    return z / (1.0f + z);
}

int main(int argc, char **argv) {
    const unsigned stride = argc > 1 ? (unsigned)atoi(argv[1]) : 1;
    float table[128];
    gdn_exp_table_fill(table);
    long n = 0, bad_exp = 0, bad_sig = 0, far = 0;
    for (unsigned long long b = 0; b < 0x100000000ull; b += stride) {
        const unsigned u = (unsigned)b;
        float x;
        memcpy(&x, &u, 4);
        if (!(x >= -110.0f && x <= 90.0f)) continue;
        ++n;
        const float e1 = gdn_expf(x, table), e2 = expf(x);
        if (memcmp(&e1, &e2, 4) != 0) {
            ++bad_exp;
            unsigned a1, a2;
            memcpy(&a1, &e1, 4);
            memcpy(&a2, &e2, 4);
            if ((a1 > a2 ? a1 - a2 : a2 - a1) > 1) ++far;
        }
        const float s1 = gdn_sigmoidf(x, table), s2 = ref_sigmoid(x);
        if (memcmp(&s1, &s2, 4) != 0) ++bad_sig;
    }
    printf("{\"n\": %ld, \"exp_mismatch\": %ld, \"exp_far\": %ld, \"sigmoid_mismatch\": %ld}\n", n, bad_exp, far,
           bad_sig);
    return 0;
}
