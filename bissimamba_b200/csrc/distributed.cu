// distributed.cu -- one process per GPU over NCCL (rebuild of the reference's
// cuda/kmamba_distributed.cu and src/kmamba_distributed.c).
//
// Batch items are independent through the scans and convnd, so ranks own
// whole items and the forward needs no exchange.  The collectives are NCCL
// over NVLink / NVSwitch: the final output gather, the weight-gradient
// all-reduce of the backward and the parameter broadcast.  The reference's
// NCCL init never distributed its unique id (cuda/kmamba_distributed.cu:46-50);
// here rank 0 sends it to the other ranks over a TCP socket.
#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <nccl.h>
#include <sys/socket.h>
#include <unistd.h>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include "kmb_common.cuh"
#include "../../include/kmamba_distributed.h"
#include "../../include/kmamba_b200.h"

namespace kmb {
int set_error(const char* msg);
int set_cuda_error(const char* where, cudaError_t e);
void* workspace(int slot, size_t bytes);
}  // namespace kmb

struct KMambaDistributedContext {
    KMambaDistributedConfig config;
    ncclComm_t comm = nullptr;
    cudaStream_t stream = nullptr;
    int device = 0;
};

namespace {

int nccl_fail(const char* where, ncclResult_t r) {
    std::string m = std::string(where) + ": " + ncclGetErrorString(r);
    return kmb::set_error(m.c_str());
}

// out[i] = scale * out[i] (the all-reduce's post-scale), or out[i] (+)= tmp[i]
__global__ void dist_scale(float* __restrict__ v, size_t n, float s) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) v[i] *= s;
}
__global__ void dist_fold(float* __restrict__ out, const float* __restrict__ tmp, size_t n, int overwrite) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = overwrite ? tmp[i] : out[i] + tmp[i];
}
unsigned blocks(size_t n) { return (unsigned)((n + 255) / 256); }

cudaStream_t pick(KMambaDistributedContext* c, void* s) { return s ? (cudaStream_t)s : c->stream; }

bool send_all(int fd, const void* p, size_t n) {
    const char* c = (const char*)p;
    while (n) {
        ssize_t k = send(fd, c, n, 0);
        if (k <= 0) return false;
        c += k;
        n -= (size_t)k;
    }
    return true;
}
bool recv_all(int fd, void* p, size_t n) {
    char* c = (char*)p;
    while (n) {
        ssize_t k = recv(fd, c, n, 0);
        if (k <= 0) return false;
        c += k;
        n -= (size_t)k;
    }
    return true;
}

}  // namespace

extern "C" {

void kmamba_distributed_split_batch(KMambaDistributedConfig* cfg, size_t batch_size, size_t total_gpus) {
    if (!cfg || total_gpus == 0) return;
    cfg->world_size = (int)total_gpus;
    const size_t per = batch_size / total_gpus, rem = batch_size % total_gpus, r = (size_t)cfg->rank;
    cfg->batch_start = r < rem ? r * (per + 1) : r * per + rem;
    cfg->batch_end = cfg->batch_start + per + (r < rem ? 1 : 0);
}

void kmamba_distributed_split_layers(KMambaDistributedConfig* cfg, size_t n_layers, size_t total_gpus) {
    if (!cfg || total_gpus == 0) return;
    cfg->world_size = (int)total_gpus;
    const size_t per = n_layers / total_gpus, rem = n_layers % total_gpus, r = (size_t)cfg->rank;
    cfg->layer_start = r < rem ? r * (per + 1) : r * per + rem;
    cfg->layer_end = cfg->layer_start + per + (r < rem ? 1 : 0);
}

int kmb_dist_exchange_id(void* id128, int world_size, int rank, const char* addr, int port) {
    if (!id128 || world_size < 1 || rank < 0 || rank >= world_size) return kmb::set_error("invalid arguments");
    if (world_size == 1) return 0;
    if (!addr) addr = getenv("MASTER_ADDR") ? getenv("MASTER_ADDR") : "127.0.0.1";
    if (port <= 0) {
        const char* e = getenv("KMB_NCCL_PORT");
        const char* mp = getenv("MASTER_PORT");
        port = e ? atoi(e) : (mp ? atoi(mp) + 1 : 29501);
    }
    sockaddr_in sa;
    memset(&sa, 0, sizeof sa);
    sa.sin_family = AF_INET;
    sa.sin_port = htons((uint16_t)port);
    if (inet_pton(AF_INET, addr, &sa.sin_addr) != 1) {
        hostent* he = gethostbyname(addr);
        if (!he) return kmb::set_error("kmb_dist_exchange_id: cannot resolve MASTER_ADDR");
        memcpy(&sa.sin_addr, he->h_addr_list[0], sizeof(sa.sin_addr));
    }
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(120);
    if (rank == 0) {
        int ls = socket(AF_INET, SOCK_STREAM, 0);
        int one = 1;
        setsockopt(ls, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
        if (ls < 0 || bind(ls, (sockaddr*)&sa, sizeof sa) != 0 || listen(ls, world_size) != 0) {
            if (ls >= 0) close(ls);
            return kmb::set_error("kmb_dist_exchange_id: cannot listen on the rendezvous port");
        }
        timeval tv{120, 0};
        setsockopt(ls, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof tv);
        int ok = 0;
        for (int i = 1; i < world_size; i++) {
            int fd = accept(ls, nullptr, nullptr);
            if (fd < 0) break;
            if (send_all(fd, id128, 128)) ok++;
            close(fd);
        }
        close(ls);
        return ok == world_size - 1 ? 0 : kmb::set_error("kmb_dist_exchange_id: not every rank connected");
    }
    for (;;) {
        int fd = socket(AF_INET, SOCK_STREAM, 0);
        if (fd >= 0 && connect(fd, (sockaddr*)&sa, sizeof sa) == 0) {
            timeval tv{120, 0};
            setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof tv);
            const bool got = recv_all(fd, id128, 128);
            close(fd);
            return got ? 0 : kmb::set_error("kmb_dist_exchange_id: short read of the id");
        }
        if (fd >= 0) close(fd);
        if (std::chrono::steady_clock::now() > deadline)
            return kmb::set_error("kmb_dist_exchange_id: rank 0 did not answer in 120 s");
        std::this_thread::sleep_for(std::chrono::milliseconds(50));
    }
}

int kmb_dist_unique_id(void* id128) {
    if (!id128) return kmb::set_error("kmb_dist_unique_id: NULL");
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
    memcpy(id128, &id, sizeof id);
    return 0;
}

KMambaDistributedContext* kmb_dist_init(const void* id128, int world_size, int rank, int device) {
    if (world_size < 1 || rank < 0 || rank >= world_size || (world_size > 1 && !id128)) {
        kmb::set_error("kmb_dist_init: invalid arguments");
        return nullptr;
    }
    auto* c = new KMambaDistributedContext();
    c->config.world_size = world_size;
    c->config.rank = rank;
    if (device >= 0 && cudaSetDevice(device) != cudaSuccess) {
        kmb::set_error("kmb_dist_init: cudaSetDevice failed");
        delete c;
        return nullptr;
    }
    cudaGetDevice(&c->device);
    c->config.local_rank = c->device;
    c->config.use_nccl = world_size > 1;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        kmb::set_error("kmb_dist_init: stream creation failed");
        delete c;
        return nullptr;
    }
    if (world_size > 1) {
        ncclUniqueId id;
        memcpy(&id, id128, sizeof id);
        // KMB_NCCL_MAX_CTAS caps the CTAs of every NCCL kernel of this communicator, so that a
        // collective overlapping a persistent scan (kmb_set_sm_reserve) fits in the SMs left free
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        if (const char* mc = getenv("KMB_NCCL_MAX_CTAS")) {
            const int v = atoi(mc);
            if (v > 0) {
                cfg.maxCTAs = v;
                cfg.minCTAs = 1;
            }
        }
        ncclResult_t r = ncclCommInitRankConfig(&c->comm, world_size, id, rank, &cfg);
        if (r != ncclSuccess) {
            nccl_fail("ncclCommInitRank", r);
            cudaStreamDestroy(c->stream);
            delete c;
            return nullptr;
        }
    }
    return c;
}

KMambaDistributedContext* kmamba_distributed_init_nccl(int world_size, int rank) {
    unsigned char id[128];
    memset(id, 0, sizeof id);
    if (world_size > 1) {
        if (rank == 0 && kmb_dist_unique_id(id)) return nullptr;
        if (kmb_dist_exchange_id(id, world_size, rank, nullptr, 0)) return nullptr;
    }
    const char* lr = getenv("LOCAL_RANK");
    return kmb_dist_init(id, world_size, rank, lr ? atoi(lr) : rank);
}

void kmamba_distributed_fini_nccl(KMambaDistributedContext* ctx) {
    if (!ctx) return;
    if (ctx->comm) ncclCommDestroy(ctx->comm);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

int kmb_dist_world_size(const KMambaDistributedContext* ctx) { return ctx ? ctx->config.world_size : 0; }
int kmb_dist_rank(const KMambaDistributedContext* ctx) { return ctx ? ctx->config.rank : -1; }

int kmb_dist_allreduce_async(KMambaDistributedContext* ctx, float* buf, size_t count, float scale, void* stream) {
    if (!ctx || (!buf && count)) return kmb::set_error("kmb_dist_allreduce_async: invalid arguments");
    cudaStream_t st = pick(ctx, stream);
    if (ctx->comm && count) {
        ncclResult_t r = ncclAllReduce(buf, buf, count, ncclFloat, ncclSum, ctx->comm, st);
        if (r != ncclSuccess) return nccl_fail("ncclAllReduce", r);
    }
    if (scale != 1.0f && count) {
        dist_scale<<<blocks(count), 256, 0, st>>>(buf, count, scale);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return kmb::set_cuda_error("dist_scale", e);
    }
    return 0;
}

int kmb_dist_allgather_async(KMambaDistributedContext* ctx, const float* send, float* recv, size_t count,
                             void* stream) {
    if (!ctx || !send || !recv) return kmb::set_error("kmb_dist_allgather_async: invalid arguments");
    cudaStream_t st = pick(ctx, stream);
    if (!ctx->comm) {
        if (send == recv) return 0;
        cudaError_t e = cudaMemcpyAsync(recv, send, count * sizeof(float), cudaMemcpyDeviceToDevice, st);
        return e == cudaSuccess ? 0 : kmb::set_cuda_error("allgather copy", e);
    }
    if (getenv("KMB_DIST_CHECK")) {
        // every rank must pass the same count (a mismatch would hang NCCL): compare max and min first
        double* chk = (double*)kmb::workspace(14, 256);
        if (!chk) return kmb::set_error("kmb_dist_allgather_async: workspace allocation failed");
        const double v[2] = {(double)count, -(double)count};
        double got[2];
        cudaMemcpyAsync(chk, v, sizeof v, cudaMemcpyHostToDevice, st);
        ncclResult_t r = ncclAllReduce(chk, chk, 2, ncclDouble, ncclMax, ctx->comm, st);
        if (r != ncclSuccess) return nccl_fail("ncclAllReduce (count check)", r);
        cudaMemcpyAsync(got, chk, sizeof got, cudaMemcpyDeviceToHost, st);
        cudaStreamSynchronize(st);
        if (got[0] != (double)count || -got[1] != (double)count)
            return kmb::set_error("kmb_dist_allgather_async: ranks passed different counts");
    }
    ncclResult_t r = ncclAllGather(send, recv, count, ncclFloat, ctx->comm, st);
    return r == ncclSuccess ? 0 : nccl_fail("ncclAllGather", r);
}

int kmb_dist_broadcast_async(KMambaDistributedContext* ctx, float* buf, size_t count, int root, void* stream) {
    if (!ctx || !buf) return kmb::set_error("kmb_dist_broadcast_async: invalid arguments");
    if (!ctx->comm) return 0;
    ncclResult_t r = ncclBroadcast(buf, buf, count, ncclFloat, root, ctx->comm, pick(ctx, stream));
    return r == ncclSuccess ? 0 : nccl_fail("ncclBroadcast", r);
}

int kmamba_allreduce_gradients_nccl(KMambaDistributedContext* ctx, float* d_gradients, size_t n_elements) {
    if (kmb_dist_allreduce_async(ctx, d_gradients, n_elements, 1.0f, nullptr)) return -1;
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    return e == cudaSuccess ? 0 : kmb::set_cuda_error("allreduce", e);
}

int kmamba_broadcast_params_nccl(KMambaDistributedContext* ctx, float* d_params, size_t n_elements) {
    if (kmb_dist_broadcast_async(ctx, d_params, n_elements, 0, nullptr)) return -1;
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    return e == cudaSuccess ? 0 : kmb::set_cuda_error("broadcast", e);
}

int kmb_dist_scannd_backward(KMambaDistributedContext* ctx, ScanNDParams* p, long local_batch, float* dx,
                             int overwrite, void* stream) {
    if (!ctx || !p || p->ndims <= 0) return kmb::set_error("kmb_dist_scannd_backward: invalid arguments");
    cudaStream_t st = pick(ctx, stream);
    const size_t nA = (size_t)p->ndims * p->D * p->M, nT = p->theta && p->dtheta ? (size_t)p->D / 2 : 0;
    // this rank's dA / dtheta go to a cleared side buffer, are summed over the ranks there,
    // then folded into the caller's buffers
    float* tmp = (float*)kmb::workspace(11, (nA + nT + 64) * sizeof(float));
    if (!tmp) return kmb::set_error("kmb_dist_scannd_backward: workspace allocation failed");
    cudaError_t e = cudaMemsetAsync(tmp, 0, (nA + nT) * sizeof(float), st);
    if (e != cudaSuccess) return kmb::set_cuda_error("memset", e);
    ScanNDParams q = *p;
    float* uA = p->dA;
    float* uT = nT ? p->dtheta : nullptr;
    q.dA = uA ? tmp : nullptr;
    q.dtheta = uT ? tmp + nA : nullptr;
    if (local_batch > 0 && scannd_backward_ex(&q, local_batch, dx, overwrite, st)) return -1;
    if (kmb_dist_allreduce_async(ctx, tmp, nA + nT, 1.0f, st)) return -1;
    if (uA) dist_fold<<<blocks(nA), 256, 0, st>>>(uA, tmp, nA, overwrite);
    if (uT) dist_fold<<<blocks(nT), 256, 0, st>>>(uT, tmp + nA, nT, overwrite);
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : kmb::set_cuda_error("dist_fold", e);
}

int kmb_dist_convnd_backward(KMambaDistributedContext* ctx, ConvNDParams* p, long local_batch, void* stream) {
    if (!ctx || !p || !p->dkernel) return kmb::set_error("kmb_dist_convnd_backward: invalid arguments");
    cudaStream_t st = pick(ctx, stream);
    long v = convnd_kernel_volume(p->ndims, p->K);
    if (local_batch > 0) {
        if (convnd_batched_async(p, local_batch, CONVND_BACKWARD, st)) return -1;
    } else {
        // no items here: contribute zeros to the sums
        cudaMemsetAsync(p->dkernel, 0, (size_t)v * p->D * sizeof(float), st);
        if (p->dbias) cudaMemsetAsync(p->dbias, 0, (size_t)p->D * sizeof(float), st);
    }
    if (kmb_dist_allreduce_async(ctx, p->dkernel, (size_t)v * p->D, 1.0f, st)) return -1;
    if (p->dbias && kmb_dist_allreduce_async(ctx, p->dbias, (size_t)p->D, 1.0f, st)) return -1;
    return 0;
}

float kmb_dist_model_train_step(KMambaDistributedContext* ctx, KMamba* m, const uint32_t* d_tokens,
                                size_t local_batch, size_t global_batch, void* stream) {
    if (!ctx || !m || global_batch == 0) {
        kmb::set_error("kmb_dist_model_train_step: invalid arguments");
        return NAN;
    }
    cudaStream_t st = pick(ctx, stream);
    size_t n = 0;
    float* g = kmb_model_grad_arena(m, &n);
    float loss = 0.0f;
    if (local_batch > 0) {
        kmb_clear_error();
        loss = kmb_model_forward_backward(m, d_tokens, local_batch, st);
        if (loss != loss && kmb_last_error()[0]) return NAN;
    } else {
        cudaMemsetAsync(g, 0, n * sizeof(float), st);
    }
    const float share = (float)local_batch / (float)global_batch;
    // gradient of the global mean loss: each rank's local mean weighted by its share, summed
    dist_scale<<<blocks(n), 256, 0, st>>>(g, n, share);
    if (kmb_dist_allreduce_async(ctx, g, n, 1.0f, st)) return NAN;
    float* lt = (float*)kmb::workspace(14, 256);
    if (!lt) {
        kmb::set_error("kmb_dist_model_train_step: workspace allocation failed");
        return NAN;
    }
    const float lw = loss * share;
    cudaMemcpyAsync(lt, &lw, sizeof(float), cudaMemcpyHostToDevice, st);
    if (kmb_dist_allreduce_async(ctx, lt, 1, 1.0f, st)) return NAN;
    if (kmb_model_optimizer_step(m, st)) return NAN;
    float out = NAN;
    cudaMemcpyAsync(&out, lt, sizeof(float), cudaMemcpyDeviceToHost, st);
    cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        kmb::set_cuda_error("kmb_dist_model_train_step", e);
        return NAN;
    }
    return out;
}

}  // extern "C"
