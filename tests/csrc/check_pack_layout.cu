// Host-only check that every packed tile layout (qw6::Fmt<F>::dst) maps the
// 16 x block_bytes raw bytes of a tile-block one-to-one onto [0, 16*BB).
// Built and run on the CPU by tests/test_abi.py.
#include <cstdio>
#include <vector>

#include "qw6_dev.cuh"

template <int F>
static int check(const char* name) {
    using M = qw6::Fmt<F>;
    std::vector<int> seen(M::TB, 0);
    for (unsigned r = 0; r < 16; r++)
        for (unsigned p = 0; p < (unsigned)M::BB; p++) {
            const unsigned d = M::dst(r, p);
            if (d >= (unsigned)M::TB || seen[d]) {
                std::printf("%s: row %u byte %u -> %u invalid or duplicate\n", name, r, p, d);
                return 1;
            }
            seen[d] = 1;
        }
    std::printf("%s: %d bytes ok\n", name, M::TB);
    return 0;
}

int main() {
    int bad = 0;
    bad |= check<QW6F_Q4_K_M>("q4_k");
    bad |= check<QW6F_Q5_K>("q5_k");
    bad |= check<QW6F_Q6_K>("q6_k");
    bad |= check<QW6F_IQ2_XXS>("iq2_xxs");
    bad |= check<QW6F_IQ2_S>("iq2_s");
    bad |= check<QW6F_IQ3_S>("iq3_s");
    if (!bad) std::printf("all layouts ok\n");
    return bad;
}
