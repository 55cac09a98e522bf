// kser.cpp -- the .ser weight format (reference libs/kser) and the k-mamba
// save / load on top of it (reference src/kmamba_ser.c), host code.
//
// The byte layout, the KSerConfig / KSerTensorEntry structs and the fp16 /
// bf16 / int8 conversions are the reference's format, so files written here
// are byte-identical to the reference writer's and files it wrote load here.
// Everything else is written from the format's description: a buffered
// writer that patches vocab_count and appends the index and checksum at
// finalize, a reader that reads the whole file once and checks the SHA-256 on
// every open, and a FIPS 180-4 SHA-256.
#include <sys/stat.h>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>
#include "../../include/kmamba.h"
#include "../../include/kmamba_ser.h"
#include "../../include/kser.h"

namespace kmb {
int set_error(const char* msg);
}

static_assert(sizeof(KSerConfig) == 96, "KSerConfig is 96 bytes in the format");
static_assert(sizeof(KSerTensorEntry) == 72, "KSerTensorEntry is 72 bytes in the format");

namespace {

const uint8_t kMagic[KSER_HEADER_SIZE] = {'S', 'E', 'R', 'E', 'N', 'I', 'T', 'Y', 0xCE, 0xB7, KSER_VERSION, 0, 0, 0, 0, 0};
constexpr size_t kInt8Header = 8;   // float scale, float zero point

// ---------------------------------------------------------------- SHA-256
struct Sha256 {
    uint32_t h[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                     0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
    uint8_t buf[64];
    size_t nbuf = 0;
    uint64_t total = 0;
    static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
    void block(const uint8_t* p) {
        // round constants: first 32 bits of the fractional parts of the cube roots of the first 64 primes
        static const uint32_t k[64] = {
            0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
            0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
            0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
            0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
            0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
            0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
            0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
            0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
        uint32_t w[64];
        for (int i = 0; i < 16; i++)
            w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
        for (int i = 16; i < 64; i++) {
            const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
        for (int i = 0; i < 64; i++) {
            const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[i] + w[i];
            const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
            hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
        }
        h[0] += a; h[1] += b; h[2] += c; h[3] += d; h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
    }
    void update(const uint8_t* p, size_t n) {
        total += n;
        while (n) {
            const size_t k = std::min(n, 64 - nbuf);
            memcpy(buf + nbuf, p, k);
            nbuf += k; p += k; n -= k;
            if (nbuf == 64) { block(buf); nbuf = 0; }
        }
    }
    void final(uint8_t out[32]) {
        const uint64_t bits = total * 8;
        const uint8_t one = 0x80, zero = 0;
        update(&one, 1);
        while (nbuf != 56) update(&zero, 1);
        uint8_t len[8];
        for (int i = 0; i < 8; i++) len[i] = (uint8_t)(bits >> (56 - 8 * i));
        update(len, 8);
        for (int i = 0; i < 8; i++)
            for (int j = 0; j < 4; j++) out[4 * i + j] = (uint8_t)(h[i] >> (24 - 8 * j));
    }
};

// ---------------------------------------------------------------- conversions (the format's)
uint16_t to_f16(float f) {
    // IEEE half by truncating the mantissa (the format's rule); flush below 2^-24, saturate to inf
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t s = x >> 31, e = (x >> 23) & 0xffu, m = x & 0x7fffffu;
    if (e == 0) return (uint16_t)(s << 15);
    if (e == 0xff) return (uint16_t)(s << 15 | 0x7c00u | (m ? 0x200u : 0u));
    const int he = (int)e - 112;   // rebias 127 -> 15
    if (he >= 31) return (uint16_t)(s << 15 | 0x7c00u);
    if (he <= 0) {
        if (he < -10) return (uint16_t)(s << 15);
        return (uint16_t)(s << 15 | (((m | 0x800000u) >> (1 - he)) >> 13));
    }
    return (uint16_t)(s << 15 | (uint32_t)he << 10 | m >> 13);
}
float from_f16(uint16_t h) {
    const uint32_t s = h >> 15, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    float v;
    if (e == 0) v = ldexpf((float)m, -24);                 // zero or subnormal: m * 2^-24, exact
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = ldexpf((float)(m | 0x400u), (int)e - 25);   // (1 + m / 1024) * 2^(e - 15), exact
    if (std::isnan(v)) {
        uint32_t x = s << 31 | 0x7f800000u | m << 13;    // keep the payload bits as the format does
        memcpy(&v, &x, 4);
        return v;
    }
    return s ? -v : v;
}
uint16_t to_bf16(float f) {
    // round to nearest, ties to even, on the upper 16 bits
    uint32_t x;
    memcpy(&x, &f, 4);
    return (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
}
float from_bf16(uint16_t h) {
    const uint32_t x = (uint32_t)h << 16;
    float f;
    memcpy(&f, &x, 4);
    return f;
}

size_t stored_bytes(uint64_t n, KSerDtype d) {
    return d == KSER_INT8 ? kInt8Header + (size_t)n : (size_t)n * kser_dtype_size(d);
}

uint64_t elems(const uint32_t shape[4]) {
    uint64_t n = 1;
    for (int i = 0; i < 4; i++)
        if (shape[i] > 0) n *= shape[i];
    return n;
}

}  // namespace

// ---------------------------------------------------------------- writer
struct KSerWriter {
    FILE* fp = nullptr;
    std::string tmp, final_path;
    bool finalized = false, tensors_started = false;
    uint32_t vocab_count = 0;
    std::vector<KSerTensorEntry> entries;
    Sha256 sha;
    uint64_t pos = 0;
    std::vector<uint8_t> head;   // header + config + vocab_count + vocab (hashed at finalize: vocab_count changes)
    bool put(const void* p, size_t n) {
        if (!tensors_started) {
            head.insert(head.end(), (const uint8_t*)p, (const uint8_t*)p + n);
        } else {
            sha.update((const uint8_t*)p, n);
        }
        pos += n;
        return fwrite(p, 1, n, fp) == n;
    }
};

extern "C" {

size_t kser_dtype_size(KSerDtype d) {
    switch (d) {
        case KSER_FP16:
        case KSER_BF16: return 2;
        case KSER_INT8: return 1;
        default: return 4;
    }
}

int kser_quantize(const float* src, void* dst, uint64_t n, KSerDtype d) {
    if (!src || !dst || n == 0) return KSER_ERR_IO;
    switch (d) {
        case KSER_FP32: memcpy(dst, src, n * 4); return KSER_OK;
        case KSER_FP16:
            for (uint64_t i = 0; i < n; i++) ((uint16_t*)dst)[i] = to_f16(src[i]);
            return KSER_OK;
        case KSER_BF16:
            for (uint64_t i = 0; i < n; i++) ((uint16_t*)dst)[i] = to_bf16(src[i]);
            return KSER_OK;
        case KSER_INT8: {
            float lo = src[0], hi = src[0];
            for (uint64_t i = 1; i < n; i++) {
                lo = src[i] < lo ? src[i] : lo;
                hi = src[i] > hi ? src[i] : hi;
            }
            const float range = hi - lo;
            const float scale = range < 1e-8f ? 1.0f : range / 255.0f, zp = lo;
            uint8_t* o = (uint8_t*)dst;
            memcpy(o, &scale, 4);
            memcpy(o + 4, &zp, 4);
            for (uint64_t i = 0; i < n; i++) {
                float v = (src[i] - zp) / scale;
                v = v < 0.0f ? 0.0f : (v > 255.0f ? 255.0f : v);
                o[kInt8Header + i] = (uint8_t)(v + 0.5f);
            }
            return KSER_OK;
        }
        default: return KSER_ERR_FORMAT;
    }
}

int kser_dequantize(const void* src, float* dst, uint64_t n, KSerDtype d) {
    if (!src || !dst || n == 0) return KSER_ERR_IO;
    switch (d) {
        case KSER_FP32: memcpy(dst, src, n * 4); return KSER_OK;
        case KSER_FP16:
            for (uint64_t i = 0; i < n; i++) dst[i] = from_f16(((const uint16_t*)src)[i]);
            return KSER_OK;
        case KSER_BF16:
            for (uint64_t i = 0; i < n; i++) dst[i] = from_bf16(((const uint16_t*)src)[i]);
            return KSER_OK;
        case KSER_INT8: {
            float scale, zp;
            memcpy(&scale, src, 4);
            memcpy(&zp, (const uint8_t*)src + 4, 4);
            const uint8_t* q = (const uint8_t*)src + kInt8Header;
            for (uint64_t i = 0; i < n; i++) dst[i] = fmaf((float)q[i], scale, zp);   // one rounding
            return KSER_OK;
        }
        default: return KSER_ERR_FORMAT;
    }
}

void kser_sha256(const uint8_t* data, size_t len, uint8_t hash[32]) {
    Sha256 s;
    s.update(data, len);
    s.final(hash);
}

KSerWriter* kser_writer_create(const char* path, const KSerConfig* cfg) {
    if (!path || !cfg) return nullptr;
    auto* w = new KSerWriter();
    w->final_path = path;
    w->tmp = std::string(path) + ".tmp";
    w->fp = fopen(w->tmp.c_str(), "wb");
    if (!w->fp) {
        delete w;
        return nullptr;
    }
    const uint32_t zero = 0;
    if (!w->put(kMagic, sizeof kMagic) || !w->put(cfg, sizeof *cfg) || !w->put(&zero, 4)) {
        fclose(w->fp);
        remove(w->tmp.c_str());
        delete w;
        return nullptr;
    }
    return w;
}

int kser_writer_add_vocab(KSerWriter* w, uint32_t id, const char* token, uint16_t len) {
    if (!w || w->finalized) return KSER_ERR_IO;
    if (w->tensors_started) return KSER_ERR_FORMAT;
    if (!token && len) return KSER_ERR_IO;
    if (!w->put(&id, 4) || !w->put(&len, 2) || (len && !w->put(token, len))) return KSER_ERR_IO;
    w->vocab_count++;
    return KSER_OK;
}

int kser_writer_add_tensor(KSerWriter* w, const char* name, const void* data, const uint32_t shape[4],
                           KSerDtype src_dtype, KSerDtype storage_dtype) {
    if (!w || w->finalized || !name || !data || !shape) return KSER_ERR_IO;
    if (!w->tensors_started) {
        // the vocabulary is complete: patch its count into the buffered head, hash it
        memcpy(w->head.data() + KSER_HEADER_SIZE + sizeof(KSerConfig), &w->vocab_count, 4);
        w->sha.update(w->head.data(), w->head.size());
        w->tensors_started = true;
    }
    const uint64_t n = elems(shape);
    KSerTensorEntry e;
    memset(&e, 0, sizeof e);
    strncpy(e.name, name, 31);
    memcpy(e.shape, shape, 16);
    e.dtype = (uint8_t)storage_dtype;
    e.offset = w->pos;
    e.size_bytes = stored_bytes(n, storage_dtype);
    if (src_dtype == storage_dtype) {
        if (!w->put(data, (size_t)n * kser_dtype_size(src_dtype))) return KSER_ERR_IO;
    } else if (src_dtype == KSER_FP32) {
        std::vector<uint8_t> q(e.size_bytes);
        if (kser_quantize((const float*)data, q.data(), n, storage_dtype) != KSER_OK) return KSER_ERR_FORMAT;
        if (!w->put(q.data(), q.size())) return KSER_ERR_IO;
    } else {
        return KSER_ERR_FORMAT;
    }
    w->entries.push_back(e);
    return KSER_OK;
}

int kser_writer_finalize(KSerWriter* w) {
    if (!w || w->finalized) return KSER_ERR_IO;
    if (!w->tensors_started) {
        memcpy(w->head.data() + KSER_HEADER_SIZE + sizeof(KSerConfig), &w->vocab_count, 4);
        w->sha.update(w->head.data(), w->head.size());
        w->tensors_started = true;
    }
    for (auto& e : w->entries)
        if (!w->put(&e, sizeof e)) return KSER_ERR_IO;
    const uint32_t tc = (uint32_t)w->entries.size();
    if (!w->put(&tc, 4)) return KSER_ERR_IO;
    // the vocab count placeholder in the file
    if (fseek(w->fp, KSER_HEADER_SIZE + (long)sizeof(KSerConfig), SEEK_SET) != 0 ||
        fwrite(&w->vocab_count, 4, 1, w->fp) != 1 || fseek(w->fp, 0, SEEK_END) != 0)
        return KSER_ERR_IO;
    uint8_t hash[32];
    w->sha.final(hash);
    if (fwrite(hash, 1, 32, w->fp) != 32 || fflush(w->fp) != 0) return KSER_ERR_IO;
    w->finalized = true;
    return KSER_OK;
}

void kser_writer_free(KSerWriter* w) {
    if (!w) return;
    if (!w->finalized && w->fp) kser_writer_finalize(w);
    if (w->fp) {
        fclose(w->fp);
        if (w->finalized) rename(w->tmp.c_str(), w->final_path.c_str());
        else remove(w->tmp.c_str());
    }
    delete w;
}

}  // extern "C"

// ---------------------------------------------------------------- reader
struct KSerReader {
    std::vector<uint8_t> bytes;
    KSerConfig cfg;
    uint32_t vocab_count = 0;
    size_t vocab_pos = 0;
    std::vector<KSerTensorEntry> entries;
    int valid = 0;
};

extern "C" {

KSerReader* kser_reader_open(const char* path) {
    if (!path) return nullptr;
    FILE* fp = fopen(path, "rb");
    if (!fp) return nullptr;
    auto* r = new KSerReader();
    fseek(fp, 0, SEEK_END);
    const long sz = ftell(fp);
    fseek(fp, 0, SEEK_SET);
    bool ok = sz >= 152;   // header + config + vocab_count + tensor_count + checksum
    if (ok) {
        r->bytes.resize((size_t)sz);
        ok = fread(r->bytes.data(), 1, (size_t)sz, fp) == (size_t)sz;
    }
    fclose(fp);
    const uint8_t* b = r->bytes.data();
    ok = ok && memcmp(b, kMagic, 11) == 0;   // name, eta, version
    if (ok) {
        memcpy(&r->cfg, b + KSER_HEADER_SIZE, sizeof r->cfg);
        memcpy(&r->vocab_count, b + KSER_HEADER_SIZE + sizeof r->cfg, 4);
        r->vocab_pos = KSER_HEADER_SIZE + sizeof r->cfg + 4;
        size_t pos = r->vocab_pos;
        for (uint32_t i = 0; ok && i < r->vocab_count; i++) {
            uint16_t len;
            if (pos + 6 > (size_t)sz) { ok = false; break; }
            memcpy(&len, b + pos + 4, 2);
            pos += 6 + len;
        }
        const size_t cks = (size_t)sz - 32;
        uint32_t tc = 0;
        if (ok && cks >= 4) memcpy(&tc, b + cks - 4, 4);
        const size_t ent = cks - 4 - (size_t)tc * sizeof(KSerTensorEntry);
        ok = ok && cks >= 4 && (size_t)tc * sizeof(KSerTensorEntry) <= cks - 4 && ent >= pos;
        if (ok) {
            r->entries.resize(tc);
            if (tc) memcpy(r->entries.data(), b + ent, (size_t)tc * sizeof(KSerTensorEntry));
            for (auto& e : r->entries)
                if (e.offset + e.size_bytes > ent) ok = false;
            uint8_t h[32];
            kser_sha256(b, cks, h);
            r->valid = memcmp(h, b + cks, 32) == 0;
        }
    }
    if (!ok) {
        delete r;
        return nullptr;
    }
    return r;
}

const KSerConfig* kser_reader_config(KSerReader* r) { return r ? &r->cfg : nullptr; }
int kser_reader_is_valid(KSerReader* r) { return r ? r->valid : 0; }

int kser_reader_load_vocab(KSerReader* r, KSerVocabCallback cb, void* userdata) {
    if (!r || !cb) return KSER_OK;
    size_t pos = r->vocab_pos;
    std::string tok;
    for (uint32_t i = 0; i < r->vocab_count; i++) {
        uint32_t id;
        uint16_t len;
        memcpy(&id, r->bytes.data() + pos, 4);
        memcpy(&len, r->bytes.data() + pos + 4, 2);
        tok.assign((const char*)r->bytes.data() + pos + 6, len);
        const int rc = cb(id, tok.c_str(), len, userdata);
        if (rc) return rc;
        pos += 6 + len;
    }
    return KSER_OK;
}

float* kser_reader_load_tensor(KSerReader* r, const char* name) {
    if (!r || !name) return nullptr;
    for (auto& e : r->entries) {
        if (strncmp(e.name, name, 32) != 0) continue;
        const uint64_t n = elems(e.shape);
        float* out = (float*)calloc(n ? n : 1, sizeof(float));
        if (!out) return nullptr;
        if (kser_dequantize(r->bytes.data() + e.offset, out, n, (KSerDtype)e.dtype) != KSER_OK) {
            free(out);
            return nullptr;
        }
        return out;
    }
    return nullptr;
}

uint64_t kser_reader_count_tensors(KSerReader* r) { return r ? r->entries.size() : 0; }
const KSerTensorEntry* kser_reader_get_tensor_info(KSerReader* r, uint64_t idx) {
    return (r && idx < r->entries.size()) ? &r->entries[idx] : nullptr;
}
void kser_reader_close(KSerReader* r) { delete r; }

KSerInfo kser_file_info(const char* path) {
    KSerInfo info;
    memset(&info, 0, sizeof info);
    if (!path) return info;
    struct stat st;
    if (stat(path, &st) == 0) info.file_size = (uint64_t)st.st_size;
    FILE* fp = fopen(path, "rb");
    if (!fp) return info;
    uint8_t hdr[KSER_HEADER_SIZE];
    KSerConfig c;
    if (fread(hdr, 1, sizeof hdr, fp) == sizeof hdr && memcmp(hdr, kMagic, 11) == 0 &&
        fread(&c, sizeof c, 1, fp) == 1) {
        info.valid = 1;
        info.vocab_size = c.vocab_size;
        info.dim = c.dim;
        info.n_layers = c.n_layers;
        info.dtype = c.dtype;
        memcpy(info.model_name, c.model_name, 64);
        // the reference's rough estimate (libs/kser/src/kser_read.c:360-363)
        info.n_params = (uint64_t)c.vocab_size * c.dim * 2 + (uint64_t)c.dim * c.state_size * 4 * c.n_layers +
                        (uint64_t)c.dim * c.dim * 4 * c.n_layers;
    }
    fclose(fp);
    return info;
}

// ---------------------------------------------------------------- k-mamba models
static const char* const kLayerFields[] = {"W_in", "W_out", "A_log", "W_B", "W_C",
                                           "delta_proj", "lambda_proj", "b_B", "b_C", "theta"};

int kmamba_save_ser(KMamba* m, const char* path, KSerDtype dtype) {
    if (!m || !path) return KSER_ERR_IO;
    const KMambaConfig* cfg = kmamba_get_config(m);
    if (!cfg) return KSER_ERR_IO;
    KSerConfig sc;
    memset(&sc, 0, sizeof sc);
    sc.vocab_size = (uint32_t)cfg->vocab_size;
    sc.dim = (uint32_t)cfg->dim;
    sc.state_size = (uint32_t)cfg->state_size;
    sc.n_layers = (uint32_t)cfg->n_layers;
    sc.seq_len = (uint32_t)cfg->seq_len;
    sc.d_conv = cfg->d_conv;
    sc.expand_factor = cfg->expand_factor;
    sc.dtype = (uint8_t)dtype;
    snprintf(sc.model_name, sizeof sc.model_name, "%s", cfg->model_name);
    KSerWriter* w = kser_writer_create(path, &sc);
    if (!w) return KSER_ERR_IO;
    const uint32_t V = sc.vocab_size, D = sc.dim, N = sc.state_size;
    const uint32_t R = cfg->mimo_rank > 1 ? (uint32_t)cfg->mimo_rank : 1, TS = N / 2 > 0 ? N / 2 : 1;
    int rc = KSER_OK;
    auto add = [&](const std::string& name, uint32_t a, uint32_t b) {
        if (rc != KSER_OK) return;
        const float* t = kmamba_get_tensor(m, name.c_str());
        const uint32_t shape[4] = {a, b, 0, 0};
        rc = t ? kser_writer_add_tensor(w, name.c_str(), t, shape, KSER_FP32, dtype) : KSER_ERR_NOT_FOUND;
    };
    add("embedding", V, D);
    for (uint32_t l = 0; l < sc.n_layers; l++) {
        const std::string p = "layers." + std::to_string(l) + ".";
        add(p + "W_in", R, D);
        add(p + "W_out", D, R);
        add(p + "A_log", N, 0);
        add(p + "W_B", N * R, D);
        add(p + "W_C", N * R, D);
        add(p + "delta_proj", D, 0);
        add(p + "lambda_proj", D, 0);
        add(p + "b_B", N * R, 0);
        add(p + "b_C", N * R, 0);
        add(p + "theta", TS, 0);
    }
    add("head", D, V);
    if (rc == KSER_OK) rc = kser_writer_finalize(w);
    kser_writer_free(w);
    return rc;
}

KMamba* kmb_load_ser_ex(const char* path, int flags, const KMambaConfig* base) {
    KSerReader* r = kser_reader_open(path);
    if (!r) {
        kmb::set_error("kmamba_load_ser: not a readable .ser file");
        return nullptr;
    }
    if ((flags & KM_SER_VERIFY) && !r->valid) {
        kmb::set_error("kmamba_load_ser: checksum mismatch");
        kser_reader_close(r);
        return nullptr;
    }
    KMambaConfig cfg;
    if (base) cfg = *base;
    else kmamba_config_set_defaults(&cfg);
    const KSerConfig& s = r->cfg;
    cfg.vocab_size = s.vocab_size;
    cfg.dim = s.dim;
    cfg.state_size = s.state_size;
    cfg.n_layers = s.n_layers;
    cfg.seq_len = s.seq_len;
    cfg.d_conv = s.d_conv;
    cfg.expand_factor = s.expand_factor;
    snprintf(cfg.model_name, sizeof cfg.model_name, "%s", s.model_name);
    for (auto& e : r->entries)
        if (!strcmp(e.name, "layers.0.W_in") && e.shape[0] > 0) cfg.mimo_rank = e.shape[0];
    if (!base) {
        cfg.spatial_ndims = 0;   // 1D over seq_len: the file has no spatial shape
    }
    KMamba* m = kmamba_create(&cfg);
    if (!m) {
        kser_reader_close(r);
        return nullptr;
    }
    for (auto& e : r->entries) {
        float* t = kser_reader_load_tensor(r, e.name);
        const int rc = t ? kmamba_set_tensor(m, e.name, t) : -1;
        free(t);
        if (rc != 0) {
            kmb::set_error((std::string("kmamba_load_ser: tensor ") + e.name + " does not fit the model").c_str());
            kmamba_free(m);
            kser_reader_close(r);
            return nullptr;
        }
    }
    kser_reader_close(r);
    return m;
}

KMamba* kmamba_load_ser(const char* path, int flags) { return kmb_load_ser_ex(path, flags, nullptr); }

KMSerInfo kmamba_ser_info(const char* path) {
    KMSerInfo info;
    memset(&info, 0, sizeof info);
    info.base = kser_file_info(path);
    info.n_layers = info.base.n_layers;
    if (info.base.valid) {
        FILE* fp = fopen(path, "rb");
        KSerConfig c;
        if (fp && fseek(fp, KSER_HEADER_SIZE, SEEK_SET) == 0 && fread(&c, sizeof c, 1, fp) == 1) {
            info.state_size = c.state_size;
            info.seq_len = c.seq_len;
        }
        if (fp) fclose(fp);
    }
    return info;
}

int kmamba_save_checkpoint_ser(KMamba* m, void* opt, const char* path, KSerDtype dtype) {
    (void)opt;
    return kmamba_save_ser(m, path, dtype);
}

int kmamba_load_checkpoint_ser(const char* path, KMamba** m_out, void** opt_out, int flags) {
    if (!path || !m_out) return KSER_ERR_IO;
    *m_out = kmamba_load_ser(path, flags);
    if (opt_out) *opt_out = nullptr;
    return *m_out ? KSER_OK : KSER_ERR_IO;
}

}  // extern "C"
