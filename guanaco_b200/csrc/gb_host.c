/*
 * gb_host.c -- host-only C11 helpers of libguanaco_b200.so.
 * Compiled as C11 (-ffp-contract=off), like the reference, so float
 * expressions round exactly as the reference's CPU code does.
 */
#include <math.h>
#include <stddef.h>

/* RoPE cos/sin table for positions [0, max_seq), restating the angle
 * computation of rope() (src/kernels/cpu/kernels_cpu.c:408-413):
 *   freq = 1 / powf(theta, i / head_dim)   (i even)
 *   angle = pos * freq,  cs = {cosf(angle), sinf(angle)}
 * Layout: h_cs[(pos * head_dim/2 + i/2) * 2 + {0,1}]. */
void gb_host_rope_table(float* h_cs, int max_seq, int head_dim, float theta) {
    const int half = head_dim / 2;
    for (int i = 0; i < head_dim; i += 2) {
        const float freq = 1.0f / powf(theta, (float)i / (float)head_dim);
        for (int pos = 0; pos < max_seq; pos++) {
            const float angle = pos * freq;
            float* o = h_cs + ((size_t)pos * half + (size_t)(i / 2)) * 2;
            o[0] = cosf(angle);
            o[1] = sinf(angle);
        }
    }
}
