// wavefront.cpp -- host wavefront skeleton (reference src/wavefront_nd.c,
// src/wavefront_plan.c): level(idx) = sum(idx), plans list row-major offsets
// grouped by level, lexicographic inside a level.  Written from the documented
// behaviour: levels are filled by one row-major sweep that buckets points by
// level (a stable bucket sort keeps lexicographic order inside each level).
#include <climits>
#include <cstdlib>
#include <cstring>
#include <vector>
#include "../../include/wavefront_plan.h"

namespace {
bool mul_ok(long a, long b, long* out) {
    if (a < 0 || b < 0) return false;
    if (a != 0 && b > LONG_MAX / a) return false;
    *out = a * b;
    return true;
}
}  // namespace

extern "C" {

int wavefront_nd_validate_dims(const long* dims, long ndims) {
    if (!dims || ndims <= 0) return 0;
    for (long i = 0; i < ndims; i++)
        if (dims[i] <= 0) return 0;
    return 1;
}

long wavefront_nd_total_points(const long* dims, long ndims) {
    if (!wavefront_nd_validate_dims(dims, ndims)) return -1;
    long t = 1;
    for (long i = 0; i < ndims; i++)
        if (!mul_ok(t, dims[i], &t)) return -1;
    return t;
}

long wavefront_nd_max_level(const long* dims, long ndims) {
    if (!wavefront_nd_validate_dims(dims, ndims)) return -1;
    long l = 0;
    for (long i = 0; i < ndims; i++) {
        if (l > LONG_MAX - (dims[i] - 1)) return -1;
        l += dims[i] - 1;
    }
    return l;
}

long wavefront_nd_row_major_offset(const long* dims, const long* idx, long ndims) {
    if (!wavefront_nd_validate_dims(dims, ndims) || !idx) return -1;
    long off = 0;
    for (long a = 0; a < ndims; a++) {
        if (idx[a] < 0 || idx[a] >= dims[a]) return -1;
        if (!mul_ok(off, dims[a], &off)) return -1;
        if (off > LONG_MAX - idx[a]) return -1;
        off += idx[a];
    }
    return off;
}

// Points of `level` whose axes >= a sum to `rem`, counted recursively.
static long count_rec(const long* dims, const long* cap, long nd, long a, long rem) {
    if (rem < 0 || rem > cap[a]) return 0;
    if (a == nd - 1) return rem < dims[a] ? 1 : 0;
    long c = 0;
    long hi = rem < dims[a] - 1 ? rem : dims[a] - 1;
    for (long v = 0; v <= hi; v++) c += count_rec(dims, cap, nd, a + 1, rem - v);
    return c;
}

static std::vector<long> suffix_caps(const long* dims, long nd) {
    std::vector<long> cap(nd + 1, 0);
    for (long a = nd - 1; a >= 0; a--) cap[a] = cap[a + 1] + dims[a] - 1;
    return cap;
}

long wavefront_nd_level_size(const long* dims, long ndims, long level) {
    long ml = wavefront_nd_max_level(dims, ndims);
    if (ml < 0 || level < 0 || level > ml) return -1;
    std::vector<long> cap = suffix_caps(dims, ndims);
    return count_rec(dims, cap.data(), ndims, 0, level);
}

struct EmitCtx {
    const long* dims;
    const long* cap;
    long nd, level, ordinal;
    long* idx;
    WavefrontNDVisitFn visit;
    void* user;
    int stop;
};

static void emit_rec(EmitCtx* c, long a, long rem) {
    if (c->stop || rem < 0 || rem > c->cap[a]) return;
    if (a == c->nd - 1) {
        if (rem < c->dims[a]) {
            c->idx[a] = rem;
            int r = c->visit(c->idx, c->nd, c->level, c->ordinal++, c->user);
            if (r != 0) c->stop = r;
        }
        return;
    }
    long hi = rem < c->dims[a] - 1 ? rem : c->dims[a] - 1;
    for (long v = 0; v <= hi && !c->stop; v++) {
        c->idx[a] = v;
        emit_rec(c, a + 1, rem - v);
    }
}

int wavefront_nd_for_level(const long* dims, long ndims, long level, long* idx_scratch,
                           WavefrontNDVisitFn visit, void* user) {
    if (!wavefront_nd_validate_dims(dims, ndims) || !visit) return -1;
    long ml = wavefront_nd_max_level(dims, ndims);
    if (ml < 0 || level < 0 || level > ml) return -1;
    std::vector<long> own;
    long* idx = idx_scratch;
    if (!idx) {
        own.assign(ndims, 0);
        idx = own.data();
    }
    std::vector<long> cap = suffix_caps(dims, ndims);
    EmitCtx c{dims, cap.data(), ndims, level, 0, idx, visit, user, 0};
    emit_rec(&c, 0, level);
    return c.stop;
}

int wavefront_nd_for_each_level(const long* dims, long ndims, long* idx_scratch,
                                WavefrontNDVisitFn visit, void* user) {
    long ml = wavefront_nd_max_level(dims, ndims);
    if (ml < 0 || !visit) return -1;
    for (long l = 0; l <= ml; l++) {
        int r = wavefront_nd_for_level(dims, ndims, l, idx_scratch, visit, user);
        if (r != 0) return r;
    }
    return 0;
}

void km_wavefront_plan_free(KMWavefrontPlan* plan) {
    if (!plan) return;
    free(plan->dims);
    free(plan->level_starts);
    free(plan->level_offsets);
    free(plan->scratch_thread);
    free(plan->coords_thread);
    free(plan);
}

KMWavefrontPlan* km_wavefront_plan_create(const long* dims, long ndims, long max_state) {
    long P = wavefront_nd_total_points(dims, ndims);
    long ml = wavefront_nd_max_level(dims, ndims);
    if (P <= 0 || ml < 0) return nullptr;
    KMWavefrontPlan* pl = (KMWavefrontPlan*)calloc(1, sizeof(KMWavefrontPlan));
    if (!pl) return nullptr;
    pl->dims = (long*)malloc(sizeof(long) * ndims);
    pl->level_starts = (long*)calloc(ml + 2, sizeof(long));
    pl->level_offsets = (long*)malloc(sizeof(long) * P);
    pl->n_threads = 1;
    pl->coords_thread = (long*)calloc(ndims, sizeof(long));
    if (max_state > 0) pl->scratch_thread = (float*)calloc(max_state, sizeof(float));
    if (!pl->dims || !pl->level_starts || !pl->level_offsets || !pl->coords_thread ||
        (max_state > 0 && !pl->scratch_thread)) {
        km_wavefront_plan_free(pl);
        return nullptr;
    }
    memcpy(pl->dims, dims, sizeof(long) * ndims);
    pl->ndims = ndims;
    pl->max_state = max_state;
    pl->total_points = P;
    pl->max_level = ml;
    // one row-major sweep: count, prefix-sum, then stable bucket fill
    std::vector<long> idx(ndims, 0), lvl(P);
    long cur = 0;
    for (long p = 0; p < P; p++) {
        lvl[p] = cur;
        pl->level_starts[cur + 1]++;
        for (long a = ndims - 1; a >= 0; a--) {
            if (++idx[a] < dims[a]) { cur++; break; }
            cur -= idx[a] - 1;
            idx[a] = 0;
        }
    }
    long mx = 0;
    for (long l = 0; l <= ml; l++) {
        if (pl->level_starts[l + 1] > mx) mx = pl->level_starts[l + 1];
        pl->level_starts[l + 1] += pl->level_starts[l];
    }
    pl->max_level_size = mx;
    std::vector<long> fill(pl->level_starts, pl->level_starts + ml + 1);
    for (long p = 0; p < P; p++) pl->level_offsets[fill[lvl[p]]++] = p;
    return pl;
}

int km_wavefront_plan_matches_dims(const KMWavefrontPlan* plan, const long* dims, long ndims) {
    if (!plan || !dims || ndims <= 0 || plan->ndims != ndims) return 0;
    for (long a = 0; a < ndims; a++)
        if (plan->dims[a] != dims[a]) return 0;
    return 1;
}

long km_wavefront_plan_level_size(const KMWavefrontPlan* plan, long level) {
    if (!plan || level < 0 || level > plan->max_level) return -1;
    return plan->level_starts[level + 1] - plan->level_starts[level];
}

const long* km_wavefront_plan_level_offsets(const KMWavefrontPlan* plan, long level) {
    if (!plan || level < 0 || level > plan->max_level) return nullptr;
    return plan->level_offsets + plan->level_starts[level];
}

int km_wavefront_plan_iter_forward(const KMWavefrontPlan* plan, KMWavefrontPlanIterCallback cb, void* ud) {
    if (!plan || !cb) return -1;
    for (long l = 0; l <= plan->max_level; l++)
        for (long i = plan->level_starts[l]; i < plan->level_starts[l + 1]; i++) cb(plan->level_offsets[i], l, ud);
    return 0;
}

int km_wavefront_plan_iter_reverse(const KMWavefrontPlan* plan, KMWavefrontPlanIterCallback cb, void* ud) {
    if (!plan || !cb) return -1;
    for (long l = plan->max_level; l >= 0; l--)
        for (long i = plan->level_starts[l]; i < plan->level_starts[l + 1]; i++) cb(plan->level_offsets[i], l, ud);
    return 0;
}

}  // extern "C"
