// Host-only check of the rANS encode step (csrc/common.cuh rans_enc_entry /
// rans_enc_update): for every precision P in 8..12, every frequency f in
// 1..2^P - 1 and a cumulative frequency with cum + f <= 2^P, the step must equal
// (x / f) * 2^P + (x mod f) + cum for boundary and pseudo-random states x in
// [1, f * 2^(32-P)), the range the encoders' renormalisation leaves.
// Built and run by tests/test_rans_enc_step.py; prints "ok" or the first mismatch.
#include <cstdio>
#include <cstdint>

#include "common.cuh"

int main() {
    uint64_t s = 0x9E3779B97F4A7C15ull;
    auto rnd = [&]() {
        s ^= s << 13; s ^= s >> 7; s ^= s << 17;
        return s;
    };
    for (uint32_t P = 8; P <= 12; P++) {
        const uint32_t M = 1u << P;
        for (uint32_t f = 1; f < M; f++) {
            const uint32_t cum = static_cast<uint32_t>(rnd() % (M - f + 1));
            const uint4 t = bsg::rans_enc_entry(f, cum, P);
            const uint64_t hi = static_cast<uint64_t>(f) << (32 - P);   // exclusive bound of x
            if (t.z != hi) {
                printf("threshold P=%u f=%u got %u want %llu\n", P, f, t.z, (unsigned long long)hi);
                return 1;
            }
            uint64_t probes[40] = {1, 2, f - 1 ? f - 1 : 1, f, f + 1ull, 2ull * f - 1, 2ull * f, hi - 1, hi - 2,
                                   hi - f, hi - f - 1, hi / 2, 0xFFFFull, 0x10000ull, (hi - 1) / f * f,
                                   (hi - 1) / f * f - 1};
            for (int k = 16; k < 40; k++) probes[k] = 1 + rnd() % (hi - 1);
            for (uint64_t x : probes) {
                if (x < 1 || x >= hi) continue;
                const uint64_t want = (x / f) * M + x % f + cum;
                const uint32_t got = bsg::rans_enc_update(static_cast<uint32_t>(x), t);
                if (want != got) {
                    printf("mismatch P=%u f=%u cum=%u x=%llu got %u want %llu\n", P, f, cum,
                           (unsigned long long)x, got, (unsigned long long)want);
                    return 1;
                }
            }
        }
    }
    printf("ok\n");
    return 0;
}
