// model.cu -- k-mamba model on the B200: embedding, n_layers Mamba-3 blocks,
// LM head, cross-entropy, exact backward and AdamW (reference src/kmamba.c,
// cuda/kmamba_kernels.cu, cuda/mamba_block.cu:424-457).
//
// All parameters live in one device arena [embedding | head | layer 0 | ...]
// with a matching gradient arena and AdamW moment arenas, so the optimizer is
// one elementwise launch over the arena and a data-parallel caller all-reduces
// one contiguous buffer.  The reference trains one sequence at a time
// (src/kmamba.c:534); here the whole batch goes through each block at once.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <random>
#include <string>
#include <vector>
#include "kmb_common.cuh"
#include "../../include/kmamba.h"
#include "../../include/kmamba_block.h"

namespace kmb {
int set_error(const char* msg);
int set_cuda_error(const char* where, cudaError_t e);
void clear_error();
void* workspace(int slot, size_t bytes);
cudaError_t mm_nt(bool bf16, long long M, long long N, long long K, const void* A, long long lda, const void* B,
                  long long ldb, float* D, long long ldd, bool accumulate, cudaStream_t st);
cudaError_t mm_tn(bool bf16, long long M, long long N, long long K, const void* A, long long lda, const void* B,
                  long long ldb, float* D, long long ldd, bool accumulate, cudaStream_t st);
cudaError_t gemm_transpose_f32(const float* in, float* out, long long R, long long Cn, long long ldi, long long ldo,
                               cudaStream_t st);
}
using namespace kmb;
enum { WS_HEAD_T = 17 };   // head^T [V, D] for the logits GEMM

struct LayerOfs {
    size_t W_in, W_out, A_log, W_B, W_C, delta_proj, lambda_proj, b_B, b_C, theta;
};

struct KMamba {
    KMambaConfig cfg;
    int dev = 0;
    long L = 0, D = 0, V = 0, N = 0, R = 0, NR = 0, TS = 0, nl = 0;
    std::vector<long> dims;
    size_t n_params = 0, n_eh = 0;  // total floats; embedding + head floats
    std::vector<LayerOfs> lo;
    float *params = nullptr, *grads = nullptr, *mom1 = nullptr, *mom2 = nullptr;
    int training = 0;
    MBOptimConfig opt{};
    float lr_eh = 1e-3f, wd_eh = 0.0f;
    size_t step = 0;
    // per-batch buffers
    size_t cap_batch = 0;
    float *hid = nullptr, *blk_act = nullptr, *logits = nullptr, *dh = nullptr, *dh2 = nullptr, *rowloss = nullptr,
          *loss = nullptr;
    uint32_t* tok = nullptr;
    size_t act_floats = 0;
    std::map<std::string, std::vector<float>> mirror;
};

static KMBlockConfig layer_cfg(const KMamba* m) {
    KMBlockConfig c;
    memset(&c, 0, sizeof c);
    c.dim = m->D; c.N = m->N; c.R = m->R; c.ndims = (long)m->dims.size(); c.dims = m->dims.data(); c.L = m->L;
    c.dt_min = m->cfg.dt_min; c.dt_max = m->cfg.dt_max; c.default_lambda = m->cfg.default_lambda;
    c.use_fast_exp = m->cfg.use_fast_exp;
    return c;
}

template <typename W, typename T>
static W layer_ptrs(T* base, const LayerOfs& o) {
    W w;
    w.W_in = base + o.W_in; w.W_out = base + o.W_out; w.A_log = base + o.A_log; w.W_B = base + o.W_B;
    w.W_C = base + o.W_C; w.delta_proj = base + o.delta_proj; w.lambda_proj = base + o.lambda_proj;
    w.b_B = base + o.b_B; w.b_C = base + o.b_C; w.theta = base + o.theta;
    return w;
}

// ------------------------------------------------------------------ kernels
__global__ void embed_gather(const float* __restrict__ emb, const uint32_t* __restrict__ tok, long long BL, int L,
                             int D, int V, float* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= BL * D) return;
    const long long row = i / D;
    const int d = (int)(i - row * D);
    const long long b = row / L, t = row - b * L;
    uint32_t k = tok[b * (L + 1) + t];
    if (k >= (uint32_t)V) k = 0;  // reference src/kmamba.c:643
    out[i] = emb[(long long)k * D + d];
}

__global__ void embed_scatter_grad(const float* __restrict__ dh, const uint32_t* __restrict__ tok, long long BL,
                                   int L, int D, int V, float* __restrict__ gemb) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= BL * D) return;
    const long long row = i / D;
    const int d = (int)(i - row * D);
    const long long b = row / L, t = row - b * L;
    uint32_t k = tok[b * (L + 1) + t];
    if (k >= (uint32_t)V) k = 0;
    atomicAdd(&gemb[(long long)k * D + d], dh[i]);
}

// One warp per row: cross-entropy against tok[t+1], dlogits = (softmax - onehot) * scale.
__global__ void softmax_xent(float* __restrict__ logits, const uint32_t* __restrict__ tok, long long BL, int L,
                             int V, float scale, float* __restrict__ rowloss) {
    const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= BL) return;
    float* lg = logits + row * V;
    const long long b = row / L, t = row - b * L;
    const uint32_t tgt = tok[b * (L + 1) + t + 1];
    float mx = -INFINITY;
    for (int v = lane; v < V; v += 32) mx = fmaxf(mx, lg[v]);
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float se = 0.0f;
    for (int v = lane; v < V; v += 32) se += expf(lg[v] - mx);
    for (int o = 16; o; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
    const float lse = mx + logf(se);
    if (lane == 0) rowloss[row] = (tgt < (uint32_t)V) ? lse - lg[tgt] : 0.0f;
    __syncwarp();
    for (int v = lane; v < V; v += 32) {
        const float p = expf(lg[v] - lse);
        lg[v] = (p - (v == (int)tgt ? 1.0f : 0.0f)) * scale;
    }
}

__global__ void sum_rows(const float* __restrict__ x, long long n, float scale, float* __restrict__ out) {
    // single block, fixed order per thread then tree: deterministic
    __shared__ float sh[256];
    float acc = 0.0f;
    for (long long i = threadIdx.x; i < n; i += 256) acc += x[i];
    sh[threadIdx.x] = acc;
    __syncthreads();
    for (int s = 128; s; s >>= 1) {
        if (threadIdx.x < s) sh[threadIdx.x] += sh[threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x == 0) *out = sh[0] * scale;
}

// AdamW over the arena (reference kernels/optimizer_f32.c:82-105):
// m = b1 m + (1-b1) g; v = b2 v + (1-b2) g^2; p = p(1 - lr wd) - lr (m/bc1) / (sqrt(v/bc2) + eps).
// Elements [0, n_eh) (embedding, head) use lr_eh / wd_eh, the rest lr / wd.
__global__ void adamw_arena(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m1,
                            float* __restrict__ m2, long long n, long long n_eh, float lr, float wd, float lr_eh,
                            float wd_eh, float b1, float b2, float eps, float bc1, float bc2) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float gi = g[i];
    const float mi = b1 * m1[i] + (1.0f - b1) * gi;
    const float vi = b2 * m2[i] + (1.0f - b2) * gi * gi;
    m1[i] = mi;
    m2[i] = vi;
    const bool eh = i < n_eh;
    const float l = eh ? lr_eh : lr, w = eh ? wd_eh : wd;
    const float mh = mi / bc1, vh = vi / bc2;
    p[i] = p[i] * (1.0f - l * w) - l * mh / (sqrtf(vh) + eps);
}

static inline unsigned nblk(long long n, int t) { return (unsigned)((n + t - 1) / t); }

// ------------------------------------------------------------------ host
static int ensure_batch(KMamba* m, size_t batch) {
    if (batch <= m->cap_batch) return 0;
    cudaFree(m->hid); cudaFree(m->blk_act); cudaFree(m->logits); cudaFree(m->dh); cudaFree(m->dh2);
    cudaFree(m->rowloss); cudaFree(m->loss); cudaFree(m->tok);
    m->hid = m->blk_act = m->logits = m->dh = m->dh2 = m->rowloss = m->loss = nullptr;
    m->tok = nullptr;
    m->cap_batch = 0;
    KMBlockConfig c = layer_cfg(m);
    m->act_floats = kmb_block_activation_floats(&c, (long)batch);
    const size_t BL = batch * m->L;
    cudaError_t e = cudaSuccess;
    if ((e = cudaMalloc(&m->hid, (size_t)(m->nl + 1) * BL * m->D * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->blk_act, (size_t)m->nl * m->act_floats * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->logits, BL * m->V * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->dh, BL * m->D * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->dh2, BL * m->D * 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->rowloss, BL * 4)) != cudaSuccess || (e = cudaMalloc(&m->loss, 4)) != cudaSuccess ||
        (e = cudaMalloc(&m->tok, batch * (m->L + 1) * 4)) != cudaSuccess)
        return set_cuda_error("model batch buffers", e);
    m->cap_batch = batch;
    return 0;
}

static int tensor_slot(KMamba* m, const char* name, size_t* off, size_t* n) {
    if (!strcmp(name, "embedding")) { *off = 0; *n = (size_t)m->V * m->D; return 0; }
    if (!strcmp(name, "head")) { *off = (size_t)m->V * m->D; *n = (size_t)m->D * m->V; return 0; }
    size_t li;
    char field[32];
    if (sscanf(name, "layers.%zu.%31s", &li, field) != 2 || li >= (size_t)m->nl) return -1;
    const LayerOfs& o = m->lo[li];
    const size_t D = m->D, R = m->R, N = m->N, NR = m->NR;
    struct { const char* k; size_t off, n; } t[] = {
        {"W_in", o.W_in, R * D}, {"W_out", o.W_out, D * R}, {"A_log", o.A_log, N}, {"W_B", o.W_B, NR * D},
        {"W_C", o.W_C, NR * D}, {"delta_proj", o.delta_proj, D}, {"lambda_proj", o.lambda_proj, D},
        {"b_B", o.b_B, NR}, {"b_C", o.b_C, NR}, {"theta", o.theta, (size_t)m->TS}};
    for (auto& e : t)
        if (!strcmp(field, e.k)) { *off = e.off; *n = e.n; return 0; }
    return -1;
}

extern "C" {

void kmamba_config_set_defaults(KMambaConfig* cfg) {
    if (!cfg) return;
    memset(cfg, 0, sizeof(*cfg));
    cfg->max_ndims = 8; cfg->max_state = 64; cfg->vocab_size = 32768; cfg->dim = 512; cfg->state_size = 64;
    cfg->seq_len = 1024; cfg->n_layers = 12; cfg->mimo_rank = 1; cfg->dt_scale = 1.0f; cfg->dt_min = 0.001f;
    cfg->dt_max = 0.1f; cfg->default_lambda = 0.5f; cfg->use_a_log_clamp = 1; cfg->a_log_min = -1e-5f;
    cfg->d_conv = 4; cfg->expand_factor = 2.0f; cfg->gpu_device = -1; cfg->weight_tying = 1;
    for (int i = 0; i < KMAMBA_CONFIG_MAX_NDIMS; i++) cfg->pad_left[i] = cfg->pad_right[i] = -1;
}

void kmamba_optim_config_set_defaults(MBOptimConfig* o) {
    if (!o) return;
    o->lr = 1e-3f; o->mu = 0.9f; o->beta2 = 0.999f; o->eps = 1e-8f; o->clip_norm = 1.0f; o->weight_decay = 0.01f;
}

KMamba* kmamba_create(const KMambaConfig* cfg) {
    if (!cfg || cfg->dim == 0 || cfg->state_size == 0 || cfg->seq_len == 0 || cfg->n_layers == 0 ||
        cfg->vocab_size == 0) {
        set_error("kmamba_create: dim, state_size, seq_len, n_layers and vocab_size are required");
        return nullptr;
    }
    if (cfg->max_ndims <= 0 || cfg->max_ndims > KMAMBA_CONFIG_MAX_NDIMS || cfg->max_state <= 0 ||
        cfg->state_size > 64) {
        set_error("kmamba_create: invalid max_ndims / max_state (state_size must be <= 64)");
        return nullptr;
    }
    KMamba* m = new KMamba();
    m->cfg = *cfg;
    if (cfg->gpu_device >= 0) cudaSetDevice(cfg->gpu_device);
    cudaGetDevice(&m->dev);
    m->L = (long)cfg->seq_len; m->D = (long)cfg->dim; m->V = (long)cfg->vocab_size; m->N = (long)cfg->state_size;
    m->R = cfg->mimo_rank > 1 ? (long)cfg->mimo_rank : 1;
    m->NR = m->N * m->R; m->TS = m->N / 2 > 0 ? m->N / 2 : 1; m->nl = (long)cfg->n_layers;
    if (cfg->spatial_ndims <= 0) {
        m->dims.push_back(m->L);
    } else {
        long prod = 1;
        for (long i = 0; i < cfg->spatial_ndims; i++) { m->dims.push_back(cfg->spatial_dims[i]); prod *= cfg->spatial_dims[i]; }
        if (prod != m->L || cfg->spatial_ndims > cfg->max_ndims) {
            set_error("kmamba_create: spatial_dims must multiply to seq_len");
            delete m;
            return nullptr;
        }
    }
    size_t o = 0;
    auto take = [&](size_t n) { size_t r = o; o += (n + 31) & ~(size_t)31; return r; };
    take((size_t)m->V * m->D);
    take((size_t)m->D * m->V);
    m->n_eh = o;
    const size_t D = m->D, R = m->R, N = m->N, NR = m->NR;
    for (long i = 0; i < m->nl; i++) {
        LayerOfs l;
        l.W_in = take(R * D); l.W_out = take(D * R); l.A_log = take(N); l.W_B = take(NR * D); l.W_C = take(NR * D);
        l.delta_proj = take(D); l.lambda_proj = take(D); l.b_B = take(NR); l.b_C = take(NR); l.theta = take(m->TS);
        m->lo.push_back(l);
    }
    m->n_params = o;
    if (cudaMalloc(&m->params, o * 4) != cudaSuccess || cudaMalloc(&m->grads, o * 4) != cudaSuccess) {
        set_error("kmamba_create: device allocation failed");
        kmamba_free(m);
        return nullptr;
    }
    cudaMemset(m->params, 0, o * 4);
    cudaMemset(m->grads, 0, o * 4);
    return m;
}

void kmamba_free(KMamba* m) {
    if (!m) return;
    cudaFree(m->params); cudaFree(m->grads); cudaFree(m->mom1); cudaFree(m->mom2);
    cudaFree(m->hid); cudaFree(m->blk_act); cudaFree(m->logits); cudaFree(m->dh); cudaFree(m->dh2);
    cudaFree(m->rowloss); cudaFree(m->loss); cudaFree(m->tok);
    delete m;
}

// ---- the reference's initialisation streams (bit for bit)
// Seeds are finalised with the SplitMix64 mixer, draws are xorshift64 (13, 7, 17)
// with 53-bit uniforms, as kernels/init_f32.c:17-45 and src/mamba_block.c:227-268.
namespace {
uint64_t init_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}
inline uint64_t init_next(uint64_t& s) {
    s ^= s << 13;
    s ^= s >> 7;
    s ^= s << 17;
    return s;
}
inline double init_u53(uint64_t& s) { return (double)(init_next(s) >> 11) * (1.0 / 9007199254740992.0); }

// embedding / head: Xavier-uniform over [-limit, limit), kmamba_init's stream
// (src/kmamba.c:458-459: seed for the embedding, seed + 1 for the head)
void init_xavier(float* w, size_t fan_in, size_t fan_out, uint32_t seed) {
    uint64_t s = init_mix((uint64_t)seed + 0x9e3779b97f4a7c15ULL);
    const float lim = sqrtf(6.0f / (float)(fan_in + fan_out));
    const float lo = -lim, span = lim - lo;
    for (size_t i = 0; i < fan_in * fan_out; i++) w[i] = fmaf((float)init_u53(s), span, lo);
}

// One block's tensors.  The reference seeds every block from its dimensions
// (dim, state_size, seq_len), not from the model seed or the layer index, so
// all layers start identical.  Order of the stream: W_in, W_out, W_B, W_C
// (each Xavier over rows + cols), theta, delta_proj, lambda_proj.
struct BlockInit {
    std::vector<float> W_in, W_out, A_log, W_B, W_C, b_B, b_C, theta, delta_proj, lambda_proj;
};
BlockInit init_block(size_t D, size_t N, size_t R, size_t L) {
    BlockInit b;
    uint64_t s = init_mix((uint64_t)D ^ ((uint64_t)N << 16) ^ ((uint64_t)L << 32) ^ 0x9e3779b97f4a7c15ULL);
    const size_t NR = N * R, TS = N / 2 > 0 ? N / 2 : 1;
    b.A_log.assign(N, -1.0f);
    auto mat = [&](std::vector<float>& v, size_t rows, size_t cols) {
        v.resize(rows * cols);
        const float scale = sqrtf(6.0f / (float)(rows + cols));
        for (auto& x : v) x = ((float)init_u53(s) * 2.0f - 1.0f) * scale;
    };
    mat(b.W_in, R, D);
    mat(b.W_out, D, R);
    mat(b.W_B, NR, D);
    mat(b.W_C, NR, D);
    b.b_B.assign(NR, 0.0f);
    b.b_C.assign(NR, 0.0f);
    b.theta.resize(TS);
    const float tsc = 2.0f * 3.14159f / (float)N;
    for (auto& x : b.theta) x = (float)init_u53(s) * tsc;
    b.delta_proj.resize(D);
    for (auto& x : b.delta_proj) x = ((float)init_u53(s) - 0.5f) * 0.02f;
    b.lambda_proj.resize(D);
    for (auto& x : b.lambda_proj) x = ((float)init_u53(s) - 0.5f) * 0.02f;
    return b;
}
const std::vector<float>* block_field(const BlockInit& b, const std::string& f) {
    if (f == "W_in") return &b.W_in;
    if (f == "W_out") return &b.W_out;
    if (f == "A_log") return &b.A_log;
    if (f == "W_B") return &b.W_B;
    if (f == "W_C") return &b.W_C;
    if (f == "b_B") return &b.b_B;
    if (f == "b_C") return &b.b_C;
    if (f == "theta") return &b.theta;
    if (f == "delta_proj") return &b.delta_proj;
    if (f == "lambda_proj") return &b.lambda_proj;
    return nullptr;
}
}  // namespace

long kmb_init_tensor(const KMambaConfig* cfg, uint32_t seed, const char* name, float* out, long n) {
    if (!cfg || !name || !out) return -1;
    const size_t V = cfg->vocab_size, D = cfg->dim, N = cfg->state_size, L = cfg->seq_len;
    const size_t R = cfg->mimo_rank > 1 ? cfg->mimo_rank : 1;
    const std::string nm(name);
    if (nm == "embedding" || nm == "head") {
        if ((size_t)n < V * D) return -1;
        if (nm == "embedding") init_xavier(out, V, D, seed);
        else init_xavier(out, D, V, seed + 1);
        return (long)(V * D);
    }
    unsigned li = 0;
    char field[32];
    if (sscanf(name, "layers.%u.%31s", &li, field) != 2 || li >= cfg->n_layers) return -1;
    const BlockInit b = init_block(D, N, R, L);
    const std::vector<float>* v = block_field(b, field);
    if (!v || (size_t)n < v->size()) return -1;
    memcpy(out, v->data(), v->size() * sizeof(float));
    return (long)v->size();
}

int kmamba_init(KMamba* m, uint32_t seed) {
    if (!m) return -1;
    std::vector<float> h(m->n_params, 0.0f);
    init_xavier(h.data(), m->V, m->D, seed);
    init_xavier(h.data() + (size_t)m->V * m->D, m->D, m->V, seed + 1);
    const BlockInit b = init_block(m->D, m->N, m->R, m->L);
    for (auto& l : m->lo) {
        const std::pair<size_t, const std::vector<float>*> parts[] = {
            {l.W_in, &b.W_in}, {l.W_out, &b.W_out}, {l.A_log, &b.A_log}, {l.W_B, &b.W_B}, {l.W_C, &b.W_C},
            {l.delta_proj, &b.delta_proj}, {l.lambda_proj, &b.lambda_proj}, {l.b_B, &b.b_B}, {l.b_C, &b.b_C},
            {l.theta, &b.theta}};
        for (auto& pr : parts) memcpy(h.data() + pr.first, pr.second->data(), pr.second->size() * sizeof(float));
    }
    cudaSetDevice(m->dev);
    cudaError_t e = cudaMemcpy(m->params, h.data(), m->n_params * 4, cudaMemcpyHostToDevice);
    return e == cudaSuccess ? 0 : set_cuda_error("kmamba_init", e);
}

int kmamba_enable_training(KMamba* m, const MBOptimConfig* opt, float lr_embed_head, float weight_decay) {
    if (!m || !opt) return -1;
    m->training = 1;
    m->opt = *opt;
    m->lr_eh = lr_embed_head;
    m->wd_eh = weight_decay;
    cudaSetDevice(m->dev);
    if (!m->mom1 && (cudaMalloc(&m->mom1, m->n_params * 4) != cudaSuccess ||
                     cudaMalloc(&m->mom2, m->n_params * 4) != cudaSuccess))
        return set_error("kmamba_enable_training: allocation failed");
    cudaMemset(m->mom1, 0, m->n_params * 4);
    cudaMemset(m->mom2, 0, m->n_params * 4);
    return 0;
}

// forward of `batch` sequences already in m->tok; leaves logits in m->logits
static int model_forward(KMamba* m, size_t batch, cudaStream_t st) {
    const long long BL = (long long)batch * m->L;
    embed_gather<<<nblk(BL * m->D, 256), 256, 0, st>>>(m->params, m->tok, BL, (int)m->L, (int)m->D, (int)m->V,
                                                       m->hid);
    KMBlockConfig c = layer_cfg(m);
    for (long i = 0; i < m->nl; i++) {
        KMBlockWeights w = layer_ptrs<KMBlockWeights>((const float*)m->params, m->lo[i]);
        if (kmb_block_forward(&c, &w, m->hid + (size_t)i * BL * m->D, m->hid + (size_t)(i + 1) * BL * m->D,
                              (long)batch, m->blk_act + (size_t)i * m->act_floats, st))
            return -1;
    }
    // logits[BL, V] = h[BL, D] . head[D, V] on the tensor cores at fp32 accuracy (3xTF32): B operand head^T
    float* hT = (float*)workspace(WS_HEAD_T, (size_t)m->V * m->D * sizeof(float));
    if (!hT) return set_error("workspace allocation failed");
    cudaError_t e = gemm_transpose_f32(m->params + (size_t)m->V * m->D, hT, m->D, m->V, m->V, m->D, st);
    if (e == cudaSuccess)
        e = mm_nt(false, BL, m->V, m->D, m->hid + (size_t)m->nl * BL * m->D, m->D, hT, m->D, m->logits, m->V, false,
                  st);
    return e == cudaSuccess ? 0 : set_cuda_error("head GEMM", e);
}

int kmamba_forward(KMamba* m, const uint32_t* tokens, float* logits_out) {
    if (!m || !tokens || !logits_out) return -1;
    cudaSetDevice(m->dev);
    if (ensure_batch(m, 1)) return -1;
    cudaStream_t st = 0;
    if (cudaMemcpy(m->tok, tokens, (size_t)m->L * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return set_error("token upload failed");
    if (model_forward(m, 1, st)) return -1;
    cudaError_t e = cudaMemcpy(logits_out, m->logits, (size_t)m->L * m->V * 4, cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? 0 : set_cuda_error("kmamba_forward", e);
}

float kmb_model_forward_backward(KMamba* m, const uint32_t* d_tokens, size_t batch, void* stream) {
    clear_error();
    if (!m || !d_tokens || batch == 0) {
        set_error("kmb_model_forward_backward: invalid arguments");
        return NAN;
    }
    cudaSetDevice(m->dev);
    if (ensure_batch(m, batch)) return NAN;
    cudaStream_t st = (cudaStream_t)stream;
    const long long BL = (long long)batch * m->L;
    if (cudaMemcpyAsync(m->tok, d_tokens, batch * (m->L + 1) * 4, cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
        set_error("token copy failed");
        return NAN;
    }
    cudaMemsetAsync(m->grads, 0, m->n_params * 4, st);
    if (model_forward(m, batch, st)) return NAN;
    const float inv = 1.0f / (float)BL;
    softmax_xent<<<nblk(BL, 8), 256, 0, st>>>(m->logits, m->tok, BL, (int)m->L, (int)m->V, inv, m->rowloss);
    sum_rows<<<1, 256, 0, st>>>(m->rowloss, BL, inv, m->loss);
    float* hN = m->hid + (size_t)m->nl * BL * m->D;
    // g_head[D, V] += h^T . dlogits ; dh[BL, D] = dlogits . head^T
    cudaError_t e = mm_tn(false, m->D, m->V, BL, hN, m->D, m->logits, m->V, m->grads + (size_t)m->V * m->D, m->V,
                          true, st);
    if (e == cudaSuccess)
        e = mm_nt(false, BL, m->D, m->V, m->logits, m->V, m->params + (size_t)m->V * m->D, m->V, m->dh, m->D, false,
                  st);
    if (e != cudaSuccess) {
        set_cuda_error("head backward GEMM", e);
        return NAN;
    }
    KMBlockConfig c = layer_cfg(m);
    for (long i = m->nl - 1; i >= 0; i--) {
        KMBlockWeights w = layer_ptrs<KMBlockWeights>((const float*)m->params, m->lo[i]);
        KMBlockGrads g = layer_ptrs<KMBlockGrads>(m->grads, m->lo[i]);
        if (kmb_block_backward(&c, &w, m->hid + (size_t)i * BL * m->D, m->dh, m->dh2, &g, (long)batch,
                               m->blk_act + (size_t)i * m->act_floats, st))
            return NAN;
        std::swap(m->dh, m->dh2);
    }
    embed_scatter_grad<<<nblk(BL * m->D, 256), 256, 0, st>>>(m->dh, m->tok, BL, (int)m->L, (int)m->D, (int)m->V,
                                                             m->grads);
    float loss = NAN;
    e = cudaMemcpyAsync(&loss, m->loss, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        set_cuda_error("kmb_model_forward_backward", e);
        return NAN;
    }
    return loss;
}

int kmb_model_optimizer_step(KMamba* m, void* stream) {
    if (!m || !m->training) return set_error("kmb_model_optimizer_step: call kmamba_enable_training first");
    cudaSetDevice(m->dev);
    m->step++;
    const float b1 = m->opt.mu, b2 = m->opt.beta2;
    const float bc1 = 1.0f - powf(b1, (float)m->step), bc2 = 1.0f - powf(b2, (float)m->step);
    adamw_arena<<<nblk((long long)m->n_params, 256), 256, 0, (cudaStream_t)stream>>>(
        m->params, m->grads, m->mom1, m->mom2, (long long)m->n_params, (long long)m->n_eh, m->opt.lr,
        m->opt.weight_decay, m->lr_eh, m->wd_eh, b1, b2, m->opt.eps, bc1, bc2);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : set_cuda_error("adamw", e);
}

float kmamba_train_batch(KMamba* m, const uint32_t* batch_tokens, size_t batch_size) {
    if (!m || !batch_tokens || batch_size == 0 || !m->training) {
        set_error("kmamba_train_batch: invalid arguments or training not enabled");
        return NAN;
    }
    if (m->opt.mu == 0.0f || m->opt.beta2 == 0.0f || m->opt.eps == 0.0f) {
        set_error("kmamba_train_batch: optimizer parameters (mu, beta2, eps) must be non-zero");
        return NAN;
    }
    cudaSetDevice(m->dev);
    if (ensure_batch(m, batch_size)) return NAN;
    uint32_t* dtok = nullptr;
    if (cudaMalloc(&dtok, batch_size * (m->L + 1) * 4) != cudaSuccess) {
        set_error("token buffer allocation failed");
        return NAN;
    }
    cudaMemcpy(dtok, batch_tokens, batch_size * (m->L + 1) * 4, cudaMemcpyHostToDevice);
    const float loss = kmb_model_forward_backward(m, dtok, batch_size, nullptr);
    cudaFree(dtok);
    if (std::isnan(loss) || kmb_model_optimizer_step(m, nullptr)) return NAN;
    cudaDeviceSynchronize();
    return loss;
}

float kmamba_train_step(KMamba* m, const uint32_t* tokens_plus1) { return kmamba_train_batch(m, tokens_plus1, 1); }
const KMambaConfig* kmamba_get_config(const KMamba* m) { return m ? &m->cfg : nullptr; }
size_t kmamba_step_count(const KMamba* m) { return m ? m->step : 0; }
void kmamba_update_lr(KMamba* m, float lb, float le) {
    if (m) { m->opt.lr = lb; m->lr_eh = le; }
}

float* kmamba_get_tensor(KMamba* m, const char* name) {
    size_t off, n;
    if (!m || !name || tensor_slot(m, name, &off, &n)) return nullptr;
    std::vector<float>& v = m->mirror[name];
    v.resize(n);
    cudaSetDevice(m->dev);
    if (cudaMemcpy(v.data(), m->params + off, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return nullptr;
    return v.data();
}

int kmamba_set_tensor(KMamba* m, const char* name, const float* data) {
    size_t off, n;
    if (!m || !name || !data || tensor_slot(m, name, &off, &n)) return -1;
    cudaSetDevice(m->dev);
    return cudaMemcpy(m->params + off, data, n * 4, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -1;
}

int kmb_model_tensor_offset(KMamba* m, const char* name, size_t* off, size_t* n) {
    if (!m || !name || !off || !n) return -1;
    return tensor_slot(m, name, off, n);
}

float* kmb_model_grad_arena(KMamba* m, size_t* n) {
    if (!m) return nullptr;
    if (n) *n = m->n_params;
    return m->grads;
}
float* kmb_model_param_arena(KMamba* m, size_t* n) {
    if (!m) return nullptr;
    if (n) *n = m->n_params;
    return m->params;
}

}  // extern "C"
