// Host-only dump of the fragment/operand maps of moe_common.cuh, checked by
// tests/test_layout.py (runs without a GPU).
#include <stdio.h>
#include "../flash_deepseek_b200/csrc/moe_common.cuh"

int main() {
    for (int m = 0; m < 16; m++)
        for (int t = 0; t < 4; t++)
            for (int j = 0; j < 4; j++) printf("q4k %d %d %d %d\n", m, t, j, q4k_k(m, t, j));
    for (int t = 0; t < 4; t++) printf("q4min %d %d\n", t, q4k_min_sub(t));
    for (int s = 0; s < 16; s++)
        for (int t = 0; t < 4; t++)
            for (int j = 0; j < 4; j++) printf("q6k %d %d %d %d\n", s, t, j, q6k_k(s, t, j));
    for (int p = 0; p < 192; p++) printf("q6r %d %d\n", p, q6r_src_byte(p));
    printf("sizes %zu %zu %zu\n", q6r_bytes(7168, 8), q4op_halves(7168), q6i_bytes(2048));
    const float probes[] = {0.0f, 1.0f, -2.5f, 65504.0f, 65520.0f, 1e-8f, 3e-7f, 6.1e-5f, 0.333333f, 1e30f};
    for (float f : probes) printf("f2h %.9g %u\n", f, (unsigned)f2h_rne_bits(f));
    printf("split %llu\n", (unsigned long long)splitmix64(12345));
    return 0;
}
