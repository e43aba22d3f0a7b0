/* Checks the quantizers' amax / 127 (kvm_quant.cuh div127: Markstein's
 * correction step with r = RN(1/127)) against IEEE single division on the
 * host, for every STRIDE-th non-negative finite float (STRIDE = 1: all of
 * them, about 30 s).  Prints the mismatch count; exit status 1 on any. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

int main(int argc, char **argv) {
    const uint32_t stride = argc > 1 ? (uint32_t)strtoul(argv[1], NULL, 10) : 1u;
    const float b = 127.0f;
    const float r = 0x1.020408p-7f;
    volatile float one = 1.0f;
    if (r != one / b) {
        printf("r is not RN(1/127)\n");
        return 1;
    }
    uint64_t checked = 0, bad = 0;
    for (uint64_t u = 0; u <= 0x7f7fffffu; u += stride) {
        const uint32_t w = (uint32_t)u;
        float a;
        memcpy(&a, &w, 4);
        volatile float va = a;
        const float ref = va / b;
        const float q0 = a * r;
        const float rem = fmaf(-q0, b, a);
        const float q1 = fmaf(rem, r, q0);
        if (memcmp(&ref, &q1, 4) != 0) ++bad;
        ++checked;
    }
    printf("checked %llu mismatches %llu\n", (unsigned long long)checked, (unsigned long long)bad);
    return bad ? 1 : 0;
}
