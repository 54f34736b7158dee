// Host-only check of rcp_div (csrc/common.cuh): floor(n / d) for every
// divisor 1..65536 against boundary numerators and a pseudo-random sweep.
// Built and run by tests/test_rcp_div.py; prints "ok" or the first mismatch.
#include <cstdio>
#include <cstdint>

#include "common.cuh"

int main() {
    uint64_t s = 0x9E3779B97F4A7C15ull;
    for (uint32_t d = 1; d <= 65536; d++) {
        const bsg::RcpDiv r = bsg::rcp_div_make(d);
        uint32_t probes[24] = {0u, 1u, d - 1, d, d + 1, 2 * d - 1, 2 * d, 0xFFFFFFFFu, 0xFFFFFFFEu, 0x80000000u,
                               0x7FFFFFFFu, 0xFFFFu, 0x10000u, 0xFFFFFFFFu / d * d, 0xFFFFFFFFu / d * d - 1};
        for (int k = 15; k < 24; k++) {
            s ^= s << 13; s ^= s >> 7; s ^= s << 17;
            probes[k] = static_cast<uint32_t>(s);
        }
        for (uint32_t n : probes) {
            const uint32_t q = bsg::rcp_div(n, r.m, r.sh1, r.sh2);
            if (q != n / d) {
                printf("mismatch d=%u n=%u got %u want %u\n", d, n, q, n / d);
                return 1;
            }
        }
    }
    printf("ok\n");
    return 0;
}
