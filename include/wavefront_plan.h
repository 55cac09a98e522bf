/* wavefront_plan.h -- host-side wavefront skeleton shared by scanND / convND.
 *
 * Same types and entry points as the reference include/wavefront_nd.h:29-60
 * and include/wavefront_plan.h:27-68 (level(idx) = sum of idx; a plan lists
 * the row-major offsets of every level, lexicographic inside a level), so code
 * that builds or walks plans keeps working.  On the B200 the kernels do not
 * consume the plan: every CTA owns whole recurrences and walks the grid in a
 * causal order computed on the device; the plan is validated against dims for
 * API fidelity.
 */
#ifndef KMB200_WAVEFRONT_PLAN_H
#define KMB200_WAVEFRONT_PLAN_H

#ifdef __cplusplus
extern "C" {
#endif

typedef int (*WavefrontNDVisitFn)(const long *idx, long ndims, long level,
                                  long ordinal_in_level, void *user);

/* reference include/wavefront_nd.h:29-60 */
int  wavefront_nd_validate_dims(const long *dims, long ndims);
long wavefront_nd_total_points(const long *dims, long ndims);
long wavefront_nd_max_level(const long *dims, long ndims);
long wavefront_nd_row_major_offset(const long *dims, const long *idx, long ndims);
long wavefront_nd_level_size(const long *dims, long ndims, long level);
int  wavefront_nd_for_level(const long *dims, long ndims, long level, long *idx_scratch,
                            WavefrontNDVisitFn visit, void *user);
int  wavefront_nd_for_each_level(const long *dims, long ndims, long *idx_scratch,
                                 WavefrontNDVisitFn visit, void *user);

typedef struct {
    long *dims;
    long ndims;
    long max_state;
    long total_points;
    long max_level;
    long max_level_size;
    long *level_starts;    /* [max_level + 2] */
    long *level_offsets;   /* [total_points], grouped by level */
    int n_threads;
    float *scratch_thread; /* [n_threads * max_state] */
    long  *coords_thread;  /* [n_threads * ndims] */
} KMWavefrontPlan;

typedef void (*KMWavefrontPlanIterCallback)(long offset, long level, void *userdata);

/* reference include/wavefront_plan.h:43-68 */
KMWavefrontPlan *km_wavefront_plan_create(const long *dims, long ndims, long max_state);
void km_wavefront_plan_free(KMWavefrontPlan *plan);
int  km_wavefront_plan_matches_dims(const KMWavefrontPlan *plan, const long *dims, long ndims);
long km_wavefront_plan_level_size(const KMWavefrontPlan *plan, long level);
const long *km_wavefront_plan_level_offsets(const KMWavefrontPlan *plan, long level);
int  km_wavefront_plan_iter_forward(const KMWavefrontPlan *plan, KMWavefrontPlanIterCallback cb, void *userdata);
int  km_wavefront_plan_iter_reverse(const KMWavefrontPlan *plan, KMWavefrontPlanIterCallback cb, void *userdata);

#ifdef __cplusplus
}
#endif
#endif
