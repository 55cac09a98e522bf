/* convnd_oracle.c -- TEST INFRASTRUCTURE ONLY (see oracle.h).
 * Restates the dense causal depthwise convND of the reference,
 * src/convnd.c:396-458 (forward) and src/convnd.c:464-531 (backward), with the
 * same tap order (kernel_linear ascending, axes unravelled last-fastest) so the
 * fp32 sums are formed in the same order. */
#include <stdlib.h>
#include <string.h>
#include "oracle.h"

#define MAXND 32

static long c_points(const long *dims, long nd) {
    long p = 1;
    for (long i = 0; i < nd; i++) p *= dims[i];
    return p;
}

static long c_volume(long nd, long K) {
    long v = 1;
    for (long i = 0; i < nd; i++) v *= K;
    return v;
}

/* Row-major source offset of tap kl for output coordinate oc, -1 if outside. */
static long c_src(long kl, const long *oc, const long *dims, const long *st, long nd, long K) {
    long src = 0;
    for (long a = nd; a-- > 0;) {
        long ka = kl % K;
        kl /= K;
        long sc = oc[a] - (K - 1 - ka);
        if (sc < 0 || sc >= dims[a]) return -1;
        src += sc * st[a];
    }
    return src;
}

static void c_prep(const ConvNDParams *p, long *st) {
    long s = 1;
    for (long a = p->ndims - 1; a >= 0; a--) { st[a] = s; s *= p->dims[a]; }
}

int oracle_convnd_fwd(const ConvNDParams *p) {
    if (!p || !p->input || !p->kernel || !p->output || !p->dims || p->ndims <= 0 ||
        p->ndims > MAXND || p->D <= 0 || p->K <= 0) return -1;
    const long nd = p->ndims, D = p->D, P = c_points(p->dims, nd), V = c_volume(nd, p->K);
    long st[MAXND], oc[MAXND];
    c_prep(p, st);
    for (long o = 0; o < P; o++) {
        for (long a = 0; a < nd; a++) oc[a] = (o / st[a]) % p->dims[a];
        for (long d = 0; d < D; d++) {
            float sum = p->bias ? p->bias[d] : 0.0f;
            for (long kl = 0; kl < V; kl++) {
                long src = c_src(kl, oc, p->dims, st, nd, p->K);
                if (src < 0) continue;
                sum += p->input[src * D + d] * p->kernel[kl * D + d];
            }
            p->output[o * D + d] = sum;
        }
    }
    return 0;
}

/* Gradients in the reference's traversal: levels descending, points of a level
 * in lexicographic order.  The float accumulation order of dinput / dkernel /
 * dbias depends on that order, so it is reproduced here. */
static long c_level(long o, const long *dims, const long *st, long nd) {
    long l = 0;
    for (long a = 0; a < nd; a++) l += (o / st[a]) % dims[a];
    return l;
}

int oracle_convnd_bwd(const ConvNDParams *p) {
    if (!p || !p->input || !p->kernel || !p->dy || !p->dinput || !p->dkernel || !p->dims ||
        p->ndims <= 0 || p->ndims > MAXND || p->D <= 0 || p->K <= 0) return -1;
    const long nd = p->ndims, D = p->D, P = c_points(p->dims, nd), V = c_volume(nd, p->K);
    long st[MAXND], oc[MAXND];
    c_prep(p, st);
    long maxl = 0;
    for (long a = 0; a < nd; a++) maxl += p->dims[a] - 1;
    memset(p->dinput, 0, sizeof(float) * (size_t)P * D);
    memset(p->dkernel, 0, sizeof(float) * (size_t)V * D);
    if (p->dbias) memset(p->dbias, 0, sizeof(float) * (size_t)D);
    /* row-major order inside a level == lexicographic order */
    for (long lv = maxl; lv >= 0; lv--) {
        for (long o = 0; o < P; o++) {
            if (c_level(o, p->dims, st, nd) != lv) continue;
            for (long a = 0; a < nd; a++) oc[a] = (o / st[a]) % p->dims[a];
            for (long d = 0; d < D; d++) {
                float g = p->dy[o * D + d];
                if (p->dbias) p->dbias[d] += g;
                for (long kl = 0; kl < V; kl++) {
                    long src = c_src(kl, oc, p->dims, st, nd, p->K);
                    if (src < 0) continue;
                    p->dkernel[kl * D + d] += g * p->input[src * D + d];
                    p->dinput[src * D + d] += g * p->kernel[kl * D + d];
                }
            }
        }
    }
    return 0;
}
