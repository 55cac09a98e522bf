// capi.cu -- the extern "C" boundary of libkmamba_b200.so.
//
// Replaces, for the scanND / convND hot path, the reference entry points
// src/scan_nd.c:29-252 (scannd_validate, scannd_ref_with_plan, scannd),
// cuda/scan_nd.cu:544-680 (om_scannd_forward/backward), src/convnd.c:396-573
// (convnd_forward_wavefront, convnd_backward_wavefront, convnd) and
// cuda/convnd.cu:258-436 (om_convnd_forward/backward).
//
// Rules of this layer:
//  * no CPU fallback: every computation runs on the current CUDA device; an
//    error returns -1 (convnd(): convnd_status() == -1) and is described by
//    kmb_last_error();
//  * pointers are classified with cudaPointerGetAttributes: all-device calls
//    run in place; all-host calls (scannd/convnd only) are staged through a
//    cached per-thread, per-device workspace; mixed calls are rejected;
//  * no allocation per call in steady state: workspaces only grow;
//  * synchronous entry points enqueue on the legacy default stream and
//    synchronise before returning (the reference is synchronous,
//    cuda/scan_nd.cu:603); the *_async entry points take a stream and do not.
#include <cstdio>
#include <cstring>
#include <map>
#include <string>
#include "kmb_common.cuh"
#include "../../include/scan_nd.h"
#include "../../include/convnd.h"
#include "../../include/kmamba_b200.h"

namespace kmb {
cudaError_t launch_scan_fwd_generic(const ScanDesc& s, cudaStream_t st);
cudaError_t launch_scan_fwd_tma(const ScanDesc& s, int* status, cudaStream_t st);
cudaError_t launch_scan_fwd_strips(const ScanDesc& s, int* status, cudaStream_t st);
size_t scan_bwd_generic_scratch_bytes(const ScanDesc& s);
size_t scan_bwd_wave_scratch_bytes(const ScanDesc& s);
cudaError_t launch_scan_bwd_wave(const ScanDesc& s, const float* dy, float* dA, float* dB, float* dC, float* ddelta,
                                 float* dlambda, float* dtheta, float* dx, void* scratch, cudaStream_t st);
cudaError_t launch_scan_bwd_strips(const ScanDesc& s, const float* dy, float* dA, float* dB, float* dC, float* ddelta,
                                   float* dlambda, float* dtheta, float* dx, int overwrite, void* scratch, int* status,
                                   cudaStream_t st);
size_t scan_bwd_strips_scratch_bytes(const ScanDesc& s);
cudaError_t launch_scan_bwd_generic(const ScanDesc& s, const float* dy, float* dA, float* dB, float* dC,
                                    float* ddelta, float* dlambda, float* dtheta, float* dx, void* scratch,
                                    cudaStream_t st);
cudaError_t launch_conv_fwd(const ConvDesc& c, const float* in, const float* ker, const float* bias, float* out,
                            cudaStream_t st);
size_t conv_bwd_scratch_bytes(const ConvDesc& c);
cudaError_t launch_conv_both(const ConvDesc& c, const float* in, const float* ker, const float* bias, float* out,
                             const float* dy, float* din, float* dker, float* dbias, void* scratch, cudaStream_t st);
cudaError_t launch_conv_bwd(const ConvDesc& c, const float* in, const float* ker, const float* dy, float* din,
                            float* dker, float* dbias, void* scratch, cudaStream_t st);
}  // namespace kmb

using namespace kmb;

namespace {

thread_local std::string tl_err;
thread_local int tl_conv_status = 0;
thread_local int tl_fast_path = -1;   // 1 = last forward used the TMA kernel, 0 = generic
thread_local int tl_bwd_path = -1;    // 2 = strips, 1 = wave, 0 = generic
int g_force_generic = -1;             // KMB_FORCE_GENERIC=1 disables the TMA path (tests)
int g_scan_ex2 = 0;
int g_sm_reserve = 0;                 // SMs the persistent grids leave free for concurrent kernels                   // 1: the 2D strip forward evaluates alpha with ex2.approx

int fail(const char* msg) {
    tl_err = msg;
    return -1;
}
int fail_cuda(const char* where, cudaError_t e) {
    tl_err = std::string(where) + ": " + cudaGetErrorString(e);
    return -1;
}

bool force_generic() {
    if (g_force_generic < 0) {
        const char* e = getenv("KMB_FORCE_GENERIC");
        g_force_generic = (e && e[0] == '1') ? 1 : 0;
    }
    return g_force_generic == 1;
}

// ---------------------------------------------------------------- workspace
enum WsSlot { WS_SCRATCH = 0, WS_STAGE = 1, WS_STATUS = 2, WS_NSLOTS = 20 };  // 3-4: blockscan, 5-10: block, 11 + 14: distributed, 12, 13, 15, 16: GEMMs
struct Ws {
    void* p = nullptr;
    size_t n = 0;
};
thread_local std::map<int, Ws> tl_ws[WS_NSLOTS];

void* ws_get(int slot, size_t bytes) {
    int dev = 0;
    if (slot < 0 || slot >= WS_NSLOTS) return nullptr;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    Ws& w = tl_ws[slot][dev];
    if (w.n < bytes) {
        if (w.p) cudaFree(w.p);
        w.p = nullptr;
        w.n = 0;
        size_t want = bytes + (bytes >> 3);  // grow with slack
        if (cudaMalloc(&w.p, want) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        w.n = want;
    }
    return w.p;
}

int* status_word() { return (int*)ws_get(WS_STATUS, 256); }
}  // namespace

namespace kmb {
// the device status word of this host thread and device (kernels record bounded-wait timeouts in it)
int* device_status() { return status_word(); }
}  // namespace kmb

namespace {

}  // namespace

namespace kmb {
void* workspace(int slot, size_t bytes) { return ws_get(slot, bytes); }
int persistent_sms(int sms) { return sms - g_sm_reserve > 1 ? sms - g_sm_reserve : 1; }
int set_error(const char* msg) { return fail(msg); }
void clear_error() { tl_err.clear(); }
int set_cuda_error(const char* where, cudaError_t e) { return fail_cuda(where, e); }
}  // namespace kmb

namespace {

// ----------------------------------------------------------- pointer kinds
enum PtrKind { PK_NULL = 0, PK_HOST = 1, PK_DEVICE = 2, PK_OTHER_DEVICE = 3 };

PtrKind ptr_kind(const void* p) {
    if (!p) return PK_NULL;
    cudaPointerAttributes a;
    cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return PK_HOST;
    }
    if (a.type == cudaMemoryTypeDevice) {
        int dev = 0;
        cudaGetDevice(&dev);
        return a.device == dev ? PK_DEVICE : PK_OTHER_DEVICE;
    }
    if (a.type == cudaMemoryTypeManaged) return PK_DEVICE;
    return PK_HOST;
}

// all non-null pointers must share one kind; returns that kind or -1
int common_kind(const void* const* ptrs, int n) {
    int k = PK_NULL;
    for (int i = 0; i < n; i++) {
        int pk = ptr_kind(ptrs[i]);
        if (pk == PK_NULL) continue;
        if (pk == PK_OTHER_DEVICE) return -1;
        if (k == PK_NULL) k = pk;
        else if (k != pk) return -1;
    }
    return k;
}

long long points_of(const long* dims, long nd) {
    long long p = 1;
    for (long i = 0; i < nd; i++) p *= dims[i];
    return p;
}

bool fill_desc(const ScanNDParams* p, long batch, ScanDesc* s) {
    if (p->ndims > KMB_MAXND) return false;
    memset(s, 0, sizeof(*s));
    s->nd = (int)p->ndims;
    if (p->D > 0x7fffffff || p->M > 0x7fffffff) return false;
    s->D = (int)p->D;
    s->M = (int)p->M;
    s->rope = p->theta != nullptr;
    s->has_lambda = p->lambda != nullptr;
    s->fast_exp = p->use_fast_exp != 0;
    s->clamp = p->use_a_log_clamp != 0;
    s->ex2 = g_scan_ex2;
    s->a_log_min = p->a_log_min;
    s->default_lambda = p->default_lambda;
    s->P = points_of(p->dims, p->ndims);
    s->batch = batch;
    long long st = 1;
    for (int a = s->nd - 1; a >= 0; a--) {
        s->dims[a] = p->dims[a];
        s->strides[a] = st;
        st *= p->dims[a];
    }
    s->x = p->x; s->A = p->A; s->B = p->B; s->C = p->C; s->delta = p->delta;
    s->theta = p->theta; s->lambda = p->lambda; s->h = p->h; s->y = p->y;
    return true;
}

int run_scan_fwd(const ScanDesc& s, cudaStream_t st) {
    cudaError_t e;
    if (!force_generic()) {
        int* status = status_word();
        if (!status) return fail("workspace allocation failed");
        if ((e = cudaMemsetAsync(status, 0, sizeof(int), st)) != cudaSuccess) return fail_cuda("memset", e);
        e = (s.nd == 2 || s.nd == 3) ? launch_scan_fwd_strips(s, status, st) : launch_scan_fwd_tma(s, status, st);
        if (e == cudaSuccess) {
            tl_fast_path = 1;
            return 0;
        }
        if (e != cudaErrorNotSupported) return fail_cuda("scan_fwd (TMA path)", e);
        cudaGetLastError();
    }
    tl_fast_path = 0;
    if ((e = launch_scan_fwd_generic(s, st)) != cudaSuccess) return fail_cuda("scan_fwd_generic", e);
    return 0;
}

int sync_and_check(cudaStream_t st) {
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return fail_cuda("synchronize", e);
    if (tl_fast_path == 1) {
        int v = 0;
        int* status = status_word();
        if (status && cudaMemcpy(&v, status, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && v != 0) {
            char buf[96];
            snprintf(buf, sizeof buf, "device wait limit exceeded (status %d)", v);
            return fail(buf);
        }
    }
    return 0;
}

bool scan_sizes(const ScanNDParams* p, long batch, size_t* sz /*[9]*/) {
    const size_t P = (size_t)points_of(p->dims, p->ndims), D = p->D, M = p->M, nd = p->ndims, b = batch;
    sz[0] = b * P * D;              // x
    sz[1] = nd * D * M;             // A
    sz[2] = b * P * D * M;          // B
    sz[3] = b * P * D * M;          // C
    sz[4] = b * nd * P * D;         // delta
    sz[5] = b * P * D * M;          // h
    sz[6] = b * P * D;              // y
    sz[7] = p->theta ? D / 2 : 0;   // theta
    sz[8] = p->lambda ? b * P : 0;  // lambda
    return true;
}

}  // namespace

extern "C" {

const char* kmb_last_error(void) { return tl_err.c_str(); }
void kmb_clear_error(void) { tl_err.clear(); }

int kmb_device_status(void* stream) {
    int* status = status_word();
    if (!status) return -1;
    if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return -1;
    int v = 0;
    if (cudaMemcpy(&v, status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (v != 0) cudaMemset(status, 0, sizeof(int));
    return v;
}
int kmb_last_forward_path(void) { return tl_fast_path; }
int kmb_last_backward_path(void) { return tl_bwd_path; }
void kmb_set_force_generic(int on) { g_force_generic = on ? 1 : 0; }
void kmb_set_scan_exp2(int on) { g_scan_ex2 = on ? 1 : 0; }
int kmb_get_scan_exp2(void) { return g_scan_ex2; }
void kmb_set_sm_reserve(int n) { g_sm_reserve = n > 0 ? n : 0; }

int scannd_validate(const ScanNDParams* p) {
    if (!p || !p->dims) return 0;
    if (p->ndims <= 0 || p->D <= 0 || p->M <= 0) return 0;
    if (!p->x || !p->A || !p->B || !p->C || !p->delta || !p->h || !p->y) return 0;
    if (!wavefront_nd_validate_dims(p->dims, p->ndims)) return 0;
    if (wavefront_nd_total_points(p->dims, p->ndims) <= 0) return 0;
    return 1;
}

int scannd_forward_async(ScanNDParams* p, long batch, void* stream) {
    if (!scannd_validate(p) || batch < 1) return fail("invalid ScanNDParams");
    const void* ptrs[] = {p->x, p->A, p->B, p->C, p->delta, p->h, p->y, p->theta, p->lambda};
    if (common_kind(ptrs, 9) != PK_DEVICE) return fail("scannd_forward_async needs device pointers");
    ScanDesc s;
    if (!fill_desc(p, batch, &s)) return fail("unsupported ndims / sizes");
    return run_scan_fwd(s, (cudaStream_t)stream);
}

// Host-pointer batches of more than kPipeMinBytes: the batch is cut into chunks of
// whole items and three device slots rotate over three streams, so the
// host-to-device copy of chunk i+1, the kernel on chunk i and the device-to-host
// copy of chunk i-1 run at the same time (the two copy directions use separate
// copy engines).  Returns 1 when the call is too small to gain from it.
static const size_t kPipeMinBytes = (size_t)256 << 20;
struct PipeStreams {
    cudaStream_t h2d = nullptr, comp = nullptr, d2h = nullptr;
    cudaEvent_t in[3] = {}, done[3] = {}, out[3] = {};
    bool ok = false;
};
static thread_local std::map<int, PipeStreams> tl_pipe;

static PipeStreams* pipe_streams() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    PipeStreams& ps = tl_pipe[dev];
    if (!ps.ok) {
        if (cudaStreamCreateWithFlags(&ps.h2d, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags(&ps.comp, cudaStreamNonBlocking) != cudaSuccess ||
            cudaStreamCreateWithFlags(&ps.d2h, cudaStreamNonBlocking) != cudaSuccess)
            return nullptr;
        for (int i = 0; i < 3; i++)
            if (cudaEventCreateWithFlags(&ps.in[i], cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&ps.done[i], cudaEventDisableTiming) != cudaSuccess ||
                cudaEventCreateWithFlags(&ps.out[i], cudaEventDisableTiming) != cudaSuccess)
                return nullptr;
        ps.ok = true;
    }
    return &ps;
}

static int scan_host_pipelined(ScanNDParams* p, long batch, const ScanDesc& s0) {
    size_t one[9];
    scan_sizes(p, 1, one);   // floats per item (A and theta are shared)
    const size_t per_item = (one[0] + one[2] + one[3] + one[4] + one[5] + one[6] + one[8]) * 4;
    if (batch < 2 || per_item * (size_t)batch < kPipeMinBytes) return 1;
    // chunk: ~1/8 of the batch, at most ~2 GB of inputs and outputs, at least one item
    long cb = batch / 8 > 0 ? batch / 8 : 1;
    while (cb > 1 && per_item * (size_t)cb > ((size_t)2 << 30)) cb--;
    PipeStreams* ps = pipe_streams();
    if (!ps) return fail("stream creation failed");
    // device: shared A / theta, then 3 slots of [x | B | C | delta | lambda | h | y] for cb items
    const int in_ids[5] = {0, 2, 3, 4, 8}, out_ids[2] = {5, 6};
    size_t soff[9] = {}, slot_bytes = 0;
    for (int k : in_ids) { soff[k] = slot_bytes; slot_bytes += (one[k] * cb * 4 + 255) & ~(size_t)255; }
    for (int k : out_ids) { soff[k] = slot_bytes; slot_bytes += (one[k] * cb * 4 + 255) & ~(size_t)255; }
    const size_t shared_bytes = ((one[1] * 4 + 255) & ~(size_t)255) + ((one[7] * 4 + 255) & ~(size_t)255);
    char* w = (char*)ws_get(WS_STAGE, shared_bytes + 3 * slot_bytes);
    if (!w) return fail("workspace allocation failed");
    float* dA = (float*)w;
    float* dth = (float*)(w + ((one[1] * 4 + 255) & ~(size_t)255));
    char* slots = w + shared_bytes;
    cudaError_t e;
    if ((e = cudaMemcpyAsync(dA, p->A, one[1] * 4, cudaMemcpyHostToDevice, ps->h2d)) != cudaSuccess)
        return fail_cuda("H2D A", e);
    if (p->theta && (e = cudaMemcpyAsync(dth, p->theta, one[7] * 4, cudaMemcpyHostToDevice, ps->h2d)) != cudaSuccess)
        return fail_cuda("H2D theta", e);
    int* status = status_word();
    if (!status) return fail("workspace allocation failed");
    if ((e = cudaMemsetAsync(status, 0, sizeof(int), ps->h2d)) != cudaSuccess) return fail_cuda("memset", e);
    const void* hin[9] = {p->x, nullptr, p->B, p->C, p->delta, nullptr, nullptr, nullptr, p->lambda};
    void* hout[9] = {nullptr, nullptr, nullptr, nullptr, nullptr, p->h, p->y, nullptr, nullptr};
    const long nch = (batch + cb - 1) / cb;
    int fast = -1;
    for (long i = 0; i < nch; i++) {
        const int sl = (int)(i % 3);
        const long b0 = i * cb, nb = (b0 + cb <= batch) ? cb : batch - b0;
        char* base = slots + (size_t)sl * slot_bytes;
        // inputs: the slot is free once its previous results have left
        if (i >= 3 && (e = cudaStreamWaitEvent(ps->h2d, ps->out[sl], 0)) != cudaSuccess) return fail_cuda("wait", e);
        for (int k : in_ids) {
            if (!hin[k] || !one[k]) continue;
            if ((e = cudaMemcpyAsync(base + soff[k], (const char*)hin[k] + one[k] * 4 * b0, one[k] * 4 * nb,
                                     cudaMemcpyHostToDevice, ps->h2d)) != cudaSuccess)
                return fail_cuda("H2D", e);
        }
        if ((e = cudaEventRecord(ps->in[sl], ps->h2d)) != cudaSuccess) return fail_cuda("event", e);
        // kernel
        if ((e = cudaStreamWaitEvent(ps->comp, ps->in[sl], 0)) != cudaSuccess) return fail_cuda("wait", e);
        ScanDesc s = s0;
        s.batch = nb;
        s.x = (const float*)(base + soff[0]);
        s.A = dA;
        s.B = (const float*)(base + soff[2]);
        s.C = (const float*)(base + soff[3]);
        s.delta = (const float*)(base + soff[4]);
        s.lambda = p->lambda ? (const float*)(base + soff[8]) : nullptr;
        s.theta = p->theta ? dth : nullptr;
        s.h = (float*)(base + soff[5]);
        s.y = (float*)(base + soff[6]);
        cudaError_t ek = cudaErrorNotSupported;
        if (!force_generic())
            ek = (s.nd == 2 || s.nd == 3) ? launch_scan_fwd_strips(s, status, ps->comp)
                                         : launch_scan_fwd_tma(s, status, ps->comp);
        if (ek == cudaSuccess) {
            fast = fast < 0 ? 1 : fast;
        } else {
            if (ek != cudaErrorNotSupported) return fail_cuda("scan_fwd (TMA path)", ek);
            cudaGetLastError();
            fast = 0;
            if ((e = launch_scan_fwd_generic(s, ps->comp)) != cudaSuccess) return fail_cuda("scan_fwd_generic", e);
        }
        if ((e = cudaEventRecord(ps->done[sl], ps->comp)) != cudaSuccess) return fail_cuda("event", e);
        // outputs
        if ((e = cudaStreamWaitEvent(ps->d2h, ps->done[sl], 0)) != cudaSuccess) return fail_cuda("wait", e);
        for (int k : out_ids) {
            if ((e = cudaMemcpyAsync((char*)hout[k] + one[k] * 4 * b0, base + soff[k], one[k] * 4 * nb,
                                     cudaMemcpyDeviceToHost, ps->d2h)) != cudaSuccess)
                return fail_cuda("D2H", e);
        }
        if ((e = cudaEventRecord(ps->out[sl], ps->d2h)) != cudaSuccess) return fail_cuda("event", e);
    }
    if ((e = cudaStreamSynchronize(ps->d2h)) != cudaSuccess) return fail_cuda("synchronize", e);
    if ((e = cudaStreamSynchronize(ps->comp)) != cudaSuccess) return fail_cuda("synchronize", e);
    tl_fast_path = fast < 0 ? 0 : fast;
    if (tl_fast_path == 1) {
        int v = 0;
        if (cudaMemcpy(&v, status, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess && v != 0) {
            char buf[96];
            snprintf(buf, sizeof buf, "device wait limit exceeded (status %d)", v);
            return fail(buf);
        }
    }
    return 0;
}

int scannd_batched(ScanNDParams* p, long batch) {
    if (!scannd_validate(p) || batch < 1) return fail("invalid ScanNDParams");
    const void* ptrs[] = {p->x, p->A, p->B, p->C, p->delta, p->h, p->y, p->theta, p->lambda};
    const int kind = common_kind(ptrs, 9);
    ScanDesc s;
    if (!fill_desc(p, batch, &s)) return fail("unsupported ndims / sizes");
    cudaStream_t st = 0;
    if (kind == PK_DEVICE) {
        if (run_scan_fwd(s, st)) return -1;
        return sync_and_check(st);
    }
    if (kind != PK_HOST) return fail("mixed host/device pointers");
    {
        // large host batches: pipeline the copies against the kernel (and each other)
        const int r = scan_host_pipelined(p, batch, s);
        if (r != 1) return r;
    }
    // host buffers: stage through the device workspace
    size_t sz[9];
    scan_sizes(p, batch, sz);
    size_t off[10];
    off[0] = 0;
    for (int i = 0; i < 9; i++) off[i + 1] = off[i] + ((sz[i] * 4 + 255) & ~(size_t)255);
    char* w = (char*)ws_get(WS_STAGE, off[9]);
    if (!w) return fail("workspace allocation failed");
    const void* src[9] = {p->x, p->A, p->B, p->C, p->delta, nullptr, nullptr, p->theta, p->lambda};
    cudaError_t e;
    for (int i = 0; i < 9; i++) {
        if (src[i] && sz[i]) {
            if ((e = cudaMemcpyAsync(w + off[i], src[i], sz[i] * 4, cudaMemcpyHostToDevice, st)) != cudaSuccess)
                return fail_cuda("H2D", e);
        }
    }
    s.x = (const float*)(w + off[0]);
    s.A = (const float*)(w + off[1]);
    s.B = (const float*)(w + off[2]);
    s.C = (const float*)(w + off[3]);
    s.delta = (const float*)(w + off[4]);
    s.h = (float*)(w + off[5]);
    s.y = (float*)(w + off[6]);
    s.theta = p->theta ? (const float*)(w + off[7]) : nullptr;
    s.lambda = p->lambda ? (const float*)(w + off[8]) : nullptr;
    if (run_scan_fwd(s, st)) return -1;
    if ((e = cudaMemcpyAsync(p->h, s.h, sz[5] * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess)
        return fail_cuda("D2H h", e);
    if ((e = cudaMemcpyAsync(p->y, s.y, sz[6] * 4, cudaMemcpyDeviceToHost, st)) != cudaSuccess)
        return fail_cuda("D2H y", e);
    return sync_and_check(st);
}

int scannd(ScanNDParams* p) { return scannd_batched(p, 1); }

int scannd_ref_with_plan(ScanNDParams* p, const KMWavefrontPlan* plan) {
    if (!scannd_validate(p)) return fail("invalid ScanNDParams");
    if (!km_wavefront_plan_matches_dims(plan, p->dims, p->ndims)) return fail("plan does not match dims");
    return scannd_batched(p, 1);
}

int om_scannd_forward(ScanNDParams* p) {
    if (!scannd_validate(p)) return fail("invalid ScanNDParams");
    if (scannd_forward_async(p, 1, nullptr)) return -1;
    return sync_and_check(0);
}

int scannd_backward_ex(ScanNDParams* p, long batch, float* dx, int overwrite, void* stream) {
    if (!scannd_validate(p) || batch < 1) return fail("invalid ScanNDParams");
    const void* ptrs[] = {p->x, p->A, p->B, p->C, p->delta, p->h, p->y, p->theta, p->lambda,
                          p->dA, p->dB, p->dC, p->ddelta, p->dlambda, p->dtheta, dx};
    if (common_kind(ptrs, 16) != PK_DEVICE) return fail("scannd backward needs device pointers");
    ScanDesc s;
    if (!fill_desc(p, batch, &s)) return fail("unsupported ndims / sizes");
    cudaStream_t st = (cudaStream_t)stream;
    float* dth = p->theta ? p->dtheta : nullptr;
    if (!force_generic()) {
        int* status = status_word();
        void* ws = ws_get(WS_SCRATCH, scan_bwd_strips_scratch_bytes(s));
        if (!ws || !status) return fail("workspace allocation failed");
        cudaError_t es = cudaMemsetAsync(status, 0, sizeof(int), st);
        if (es != cudaSuccess) return fail_cuda("memset", es);
        es = launch_scan_bwd_strips(s, p->y, p->dA, p->dB, p->dC, p->ddelta, p->dlambda, dth, dx,
                                                overwrite ? 1 : 0, ws, status, st);
        if (es == cudaSuccess) {
            tl_bwd_path = 2;
            return 0;
        }
        if (es != cudaErrorNotSupported) return fail_cuda("scan_bwd_strips", es);
        cudaGetLastError();
    }
    if (overwrite) {
        // the other kernels accumulate: clear the outputs first
        const size_t P = (size_t)s.P, D = s.D, M = s.M, nd = s.nd, b = batch;
        struct { void* p; size_t n; } outs[] = {{p->dA, nd * D * M}, {p->dB, b * P * D * M}, {p->dC, b * P * D * M},
                                                {p->ddelta, b * nd * P * D}, {p->dlambda, b * P},
                                                {dth, D / 2}, {dx, b * P * D}};
        for (auto& o : outs)
            if (o.p) {
                cudaError_t e = cudaMemsetAsync(o.p, 0, o.n * sizeof(float), st);
                if (e != cudaSuccess) return fail_cuda("memset", e);
            }
    }
    if (!force_generic()) {
        void* ws = ws_get(WS_SCRATCH, scan_bwd_wave_scratch_bytes(s));
        if (!ws) return fail("workspace allocation failed");
        cudaError_t ew = launch_scan_bwd_wave(s, p->y, p->dA, p->dB, p->dC, p->ddelta, p->dlambda, dth, dx, ws, st);
        if (ew == cudaSuccess) {
            tl_bwd_path = 1;
            return 0;
        }
        if (ew != cudaErrorNotSupported) return fail_cuda("scan_bwd_wave", ew);
        cudaGetLastError();
    }
    void* scratch = ws_get(WS_SCRATCH, scan_bwd_generic_scratch_bytes(s));
    if (!scratch) return fail("workspace allocation failed");
    cudaError_t e = launch_scan_bwd_generic(s, p->y, p->dA, p->dB, p->dC, p->ddelta, p->dlambda, dth, dx, scratch, st);
    if (e != cudaSuccess) return fail_cuda("scan_bwd", e);
    tl_bwd_path = 0;
    return 0;
}

int scannd_backward_async(ScanNDParams* p, long batch, float* dx, void* stream) {
    return scannd_backward_ex(p, batch, dx, 0, stream);
}

int scannd_backward_batched(ScanNDParams* p, long batch, float* dx) {
    if (scannd_backward_async(p, batch, dx, nullptr)) return -1;
    tl_fast_path = tl_bwd_path == 2 ? 1 : 0;   // the strips kernel records bounded-wait timeouts
    return sync_and_check(0);
}

int om_scannd_backward(ScanNDParams* p) { return scannd_backward_batched(p, 1, nullptr); }

// ------------------------------------------------------------------ convnd
long convnd_kernel_volume(long ndims, long K) {
    if (ndims <= 0 || K <= 0) return 0;
    long v = 1;
    for (long i = 0; i < ndims; i++) v *= K;
    return v;
}

int convnd_status(void) { return tl_conv_status; }

static bool conv_desc(const ConvNDParams* p, long batch, ConvDesc* c) {
    if (!p || !p->dims || p->ndims <= 0 || p->ndims > KMB_MAXND || p->D <= 0 || p->K <= 0) return false;
    if (!wavefront_nd_validate_dims(p->dims, p->ndims)) return false;
    memset(c, 0, sizeof(*c));
    c->nd = (int)p->ndims;
    c->D = (int)p->D;
    c->K = (int)p->K;
    long long v = 1;   // K^ndims, rejected before it can overflow an int
    for (long i = 0; i < p->ndims; i++) {
        if (v > 0x7fffffffLL / p->K) return false;
        v *= p->K;
    }
    c->V = (int)v;
    c->P = points_of(p->dims, p->ndims);
    c->batch = batch;
    long long st = 1;
    for (int a = c->nd - 1; a >= 0; a--) {
        c->dims[a] = p->dims[a];
        c->strides[a] = st;
        st *= p->dims[a];
    }
    return true;
}

int convnd_batched_async(ConvNDParams* p, long batch, int mode, void* stream) {
    ConvDesc c;
    if (batch < 1 || !conv_desc(p, batch, &c)) return fail("invalid ConvNDParams");
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    if ((mode & CONVND_FORWARD) && (mode & CONVND_BACKWARD) && p->input && p->kernel && p->output && p->dy &&
        p->dinput && p->dkernel) {
        // forward and backward together: one pass over input and dy when the fused kernel takes the shape
        const void* ptrs[] = {p->input, p->kernel, p->bias, p->output, p->dy, p->dinput, p->dkernel, p->dbias};
        if (common_kind(ptrs, 8) != PK_DEVICE) return fail("convnd needs device pointers");
        void* scratch = ws_get(WS_SCRATCH, conv_bwd_scratch_bytes(c));
        if (!scratch) return fail("workspace allocation failed");
        if ((e = launch_conv_both(c, p->input, p->kernel, p->bias, p->output, p->dy, p->dinput, p->dkernel, p->dbias,
                                  scratch, st)) != cudaSuccess)
            return fail_cuda("conv_fwd_bwd", e);
        return 0;
    }
    if (mode & CONVND_FORWARD) {
        if (!p->input || !p->kernel || !p->output) return fail("convnd forward needs input, kernel, output");
        const void* ptrs[] = {p->input, p->kernel, p->bias, p->output};
        if (common_kind(ptrs, 4) != PK_DEVICE) return fail("convnd needs device pointers");
        if ((e = launch_conv_fwd(c, p->input, p->kernel, p->bias, p->output, st)) != cudaSuccess)
            return fail_cuda("conv_fwd", e);
    }
    if (mode & CONVND_BACKWARD) {
        if (!p->input || !p->kernel || !p->dy || !p->dinput || !p->dkernel)
            return fail("convnd backward needs input, kernel, dy, dinput, dkernel");
        const void* ptrs[] = {p->input, p->kernel, p->dy, p->dinput, p->dkernel, p->dbias};
        if (common_kind(ptrs, 6) != PK_DEVICE) return fail("convnd needs device pointers");
        void* scratch = ws_get(WS_SCRATCH, conv_bwd_scratch_bytes(c));
        if (!scratch) return fail("workspace allocation failed");
        if ((e = launch_conv_bwd(c, p->input, p->kernel, p->dy, p->dinput, p->dkernel, p->dbias, scratch, st)) !=
            cudaSuccess)
            return fail_cuda("conv_bwd", e);
    }
    return 0;
}

static int convnd_sync(ConvNDParams* p, int mode) {
    ConvDesc c;
    if (!conv_desc(p, 1, &c)) return fail("invalid ConvNDParams");
    const void* ptrs[] = {p->input, p->kernel, p->bias, p->output, p->dy, p->dinput, p->dkernel, p->dbias};
    const int kind = common_kind(ptrs, 8);
    if (kind == PK_DEVICE) {
        if (convnd_batched_async(p, 1, mode, nullptr)) return -1;
        cudaError_t e = cudaStreamSynchronize(0);
        return e == cudaSuccess ? 0 : fail_cuda("synchronize", e);
    }
    if (kind != PK_HOST) return fail("mixed host/device pointers");
    const size_t PD = (size_t)c.P * c.D, VD = (size_t)c.V * c.D, D = c.D;
    // slots: input kernel bias output dy dinput dkernel dbias
    const size_t sz[8] = {PD, VD, D, PD, PD, PD, VD, D};
    size_t off[9];
    off[0] = 0;
    for (int i = 0; i < 8; i++) off[i + 1] = off[i] + ((sz[i] * 4 + 255) & ~(size_t)255);
    char* w = (char*)ws_get(WS_STAGE, off[8]);
    if (!w) return fail("workspace allocation failed");
    cudaError_t e;
    const void* hsrc[8] = {p->input, p->kernel, p->bias, nullptr, (mode & 2) ? p->dy : nullptr, nullptr, nullptr,
                           nullptr};
    for (int i = 0; i < 8; i++)
        if (hsrc[i] && (e = cudaMemcpyAsync(w + off[i], hsrc[i], sz[i] * 4, cudaMemcpyHostToDevice, 0)) != cudaSuccess)
            return fail_cuda("H2D", e);
    ConvNDParams q = *p;
    q.input = p->input ? (float*)(w + off[0]) : nullptr;
    q.kernel = p->kernel ? (const float*)(w + off[1]) : nullptr;
    q.bias = p->bias ? (const float*)(w + off[2]) : nullptr;
    q.output = p->output ? (float*)(w + off[3]) : nullptr;
    q.dy = p->dy ? (float*)(w + off[4]) : nullptr;
    q.dinput = p->dinput ? (float*)(w + off[5]) : nullptr;
    q.dkernel = p->dkernel ? (float*)(w + off[6]) : nullptr;
    q.dbias = p->dbias ? (float*)(w + off[7]) : nullptr;
    if (convnd_batched_async(&q, 1, mode, nullptr)) return -1;
    float* outs[4] = {p->output, p->dinput, p->dkernel, p->dbias};
    const int oslot[4] = {3, 5, 6, 7};
    const int omode[4] = {1, 2, 2, 2};
    for (int i = 0; i < 4; i++)
        if (outs[i] && (mode & omode[i]) &&
            (e = cudaMemcpyAsync(outs[i], w + off[oslot[i]], sz[oslot[i]] * 4, cudaMemcpyDeviceToHost, 0)) !=
                cudaSuccess)
            return fail_cuda("D2H", e);
    e = cudaStreamSynchronize(0);
    return e == cudaSuccess ? 0 : fail_cuda("synchronize", e);
}

void convnd(ConvNDParams* p, ConvNDMode mode) { tl_conv_status = convnd_sync(p, (int)mode); }

void convnd_forward_wavefront(ConvNDParams* p, const KMWavefrontPlan* plan) {
    if (!p || !km_wavefront_plan_matches_dims(plan, p->dims, p->ndims)) {
        tl_conv_status = fail("plan does not match dims");
        return;
    }
    tl_conv_status = convnd_sync(p, CONVND_FORWARD);
}

void convnd_backward_wavefront(ConvNDParams* p, const KMWavefrontPlan* plan) {
    if (!p || !km_wavefront_plan_matches_dims(plan, p->dims, p->ndims)) {
        tl_conv_status = fail("plan does not match dims");
        return;
    }
    tl_conv_status = convnd_sync(p, CONVND_BACKWARD);
}

int om_convnd_forward(ConvNDParams* p) {
    if (convnd_batched_async(p, 1, CONVND_FORWARD, nullptr)) return -1;
    cudaError_t e = cudaStreamSynchronize(0);
    return e == cudaSuccess ? 0 : fail_cuda("synchronize", e);
}

int om_convnd_backward(ConvNDParams* p) {
    if (convnd_batched_async(p, 1, CONVND_BACKWARD, nullptr)) return -1;
    cudaError_t e = cudaStreamSynchronize(0);
    return e == cudaSuccess ? 0 : fail_cuda("synchronize", e);
}

}  // extern "C"
