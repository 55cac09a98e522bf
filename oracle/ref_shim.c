/* ref_shim.c -- test infrastructure, linked ONLY into oracle/_ref/libkmamba_ref.so
 * together with the reference's own CPU sources (compiled in place).
 *
 * Purpose: call the reference's scannd_ref() safely and time it.
 *
 * The reference RoPE path (src/scan_nd.c:68-77) sizes its h_rot scratch as
 * D*M floats but indexes it with prev_offset*D*M+dm (src/scan_nd.c:159,190),
 * i.e. it needs P*D*M floats.  h_rot comes from the thread-local first-fit pool
 * (src/km_memory_pool.c:56-94).  Pre-warming that pool with two chunks of
 * >= P*D*M*4 bytes makes the first two allocations of scannd_ref_with_plan
 * (strides, then h_rot) land in those large chunks, so the reference runs
 * in-bounds with its own arithmetic unchanged.
 */
#include <stdlib.h>
#include <string.h>
#include <omp.h>
#include "scan_nd.h"
#include "convnd.h"
#include "km_memory_pool.h"
#include "wavefront_plan.h"

static long shim_points(const long *dims, long ndims) {
    long p = 1;
    for (long i = 0; i < ndims; i++) p *= dims[i];
    return p;
}

static void shim_prewarm(const ScanNDParams *p) {
    size_t big = (size_t)shim_points(p->dims, p->ndims) * (size_t)p->D * (size_t)p->M * sizeof(float);
    KMMemoryPool *pool;
    void *a, *b;
    km_memory_pool_destroy_all_threadlocal();
    pool = km_memory_pool_threadlocal();
    a = km_pool_alloc(pool, big);
    b = km_pool_alloc(pool, big);
    km_pool_free(pool, a);
    km_pool_free(pool, b);
}

/* scannd_ref() with the pool pre-warm applied (safe with theta != NULL). */
int shim_scannd_ref(ScanNDParams *p) {
    if (p && p->dims && p->ndims > 0 && p->theta) shim_prewarm(p);
    return scannd_ref(p);
}

/* Batch = a serial loop of independent reference calls (the reference API has
 * no batch dimension).  Per-item tensors are contiguous [batch, ...]; A and
 * theta are shared.  Returns the first non-zero rc. */
int shim_scannd_ref_batched(const ScanNDParams *p0, long batch) {
    long P = shim_points(p0->dims, p0->ndims);
    long D = p0->D, M = p0->M, nd = p0->ndims;
    for (long b = 0; b < batch; b++) {
        ScanNDParams p = *p0;
        p.x = p0->x + (size_t)b * P * D;
        p.B = p0->B + (size_t)b * P * D * M;
        p.C = p0->C + (size_t)b * P * D * M;
        p.delta = p0->delta + (size_t)b * nd * P * D;
        p.h = p0->h + (size_t)b * P * D * M;
        p.y = p0->y + (size_t)b * P * D;
        if (p0->lambda) p.lambda = p0->lambda + (size_t)b * P;
        int rc = shim_scannd_ref(&p);
        if (rc) return rc;
    }
    return 0;
}

/* Dense convnd forward / backward through the reference's wavefront entries
 * (src/convnd.c:396-531) with an explicit plan, i.e. the CPU path of convnd()
 * without its GPU auto-dispatch. */
int shim_convnd(ConvNDParams *p, int mode) {
    KMWavefrontPlan *plan = km_wavefront_plan_create(p->dims, p->ndims, 0);
    if (!plan) return -1;
    if (mode & 1) convnd_forward_wavefront(p, plan);
    if (mode & 2) convnd_backward_wavefront(p, plan);
    km_wavefront_plan_free(plan);
    return 0;
}

int shim_set_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
}
