// Host-only dump of the operand and repack maps of moe_common.cuh, checked by
// tests/test_layout.py (runs without a GPU).
#include <stdio.h>
#include "../flash_deepseek_b200/csrc/moe_common.cuh"

int main() {
    for (int k = 0; k < 256; k++) printf("opq4 %d %d\n", k, opq4_off(k));
    for (int k = 0; k < 256; k++) printf("opq6 %d %d\n", k, opq6_off(k));
    for (int jj = 0; jj < 16; jj++) printf("xsum %d %d\n", jj, opq4_xsum_off(jj));
    for (int k = 0; k < 256; k++) printf("opw4 %d %d\n", k, opw4_idx(k));
    for (int k = 0; k < 256; k++) printf("opw6 %d %d\n", k, opw6_idx(k));
    printf("opw %d %d %d %d %d\n", OPW_SB, OPW_XSUM, OPW_SCALE, OPW_LO, OPW_TOP);
    for (int p = 0; p < 128; p++) printf("q4r %d %d\n", p, q4r_src_qs(p));
    for (int p = 0; p < 192; p++) printf("q6r %d %d\n", p, q6r_src_byte(p));
    printf("sizes %zu %zu %zu %d %d\n", q6r_bytes(7168, 8), op_bytes(7168), op_bytes(2048), OPB_SB, OPB_PLANE);
    const float probes[] = {0.0f, 1.0f, -2.5f, 65504.0f, 65520.0f, 1e-8f, 3e-7f, 6.1e-5f, 0.333333f, 1e30f};
    for (float f : probes) printf("f2h %.9g %u\n", f, (unsigned)f2h_rne_bits(f));
    printf("split %llu\n", (unsigned long long)splitmix64(12345));
    return 0;
}
