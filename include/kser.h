/* kser.h -- the .ser weight format of the reference (libs/kser/include/kser.h),
 * implemented in libkmamba_b200.so (csrc/kser.cpp).  Same structs, enums and
 * function names, so a caller of the reference's libkser links unchanged; the
 * file bytes are the reference writer's, byte for byte.
 *
 * File layout as written (the reference's kser_write.c order):
 *   [0]    16 B  magic "SERENITY", 0xCE 0xB7 (eta), version 0x01, 5 zero bytes
 *   [16]   96 B  KSerConfig
 *   [112]   4 B  vocab_count
 *   [116]        vocab entries (id:u32, len:u16, bytes)
 *                tensor data (absolute offsets in the entries)
 *                KSerTensorEntry[tensor_count]
 *                tensor_count (u32)
 *   [end-32] 32 B SHA-256 of every preceding byte */
#ifndef KMB200_KSER_H
#define KMB200_KSER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KSER_MAGIC_SIZE 8
#define KSER_HEADER_SIZE 16
#define KSER_VERSION 0x01

typedef enum { KSER_FP32 = 0, KSER_FP16 = 1, KSER_BF16 = 2, KSER_INT8 = 3 } KSerDtype;

typedef enum {
    KSER_OK = 0,
    KSER_ERR_IO = -1,
    KSER_ERR_FORMAT = -2,
    KSER_ERR_MEMORY = -3,
    KSER_ERR_CHECKSUM = -4,
    KSER_ERR_NOT_FOUND = -5,
} KSerError;

/* 96 bytes (reference kser.h:52-63) */
typedef struct {
    uint32_t vocab_size;
    uint32_t dim;
    uint32_t state_size;
    uint32_t n_layers;
    uint32_t seq_len;
    uint32_t d_conv;
    float expand_factor;
    uint8_t dtype;
    uint8_t _pad[3];
    char model_name[64];
} KSerConfig;

/* 72 bytes (reference kser.h:66-74) */
typedef struct {
    char name[32];
    uint32_t shape[4];
    uint8_t dtype;
    uint8_t _pad[7];
    uint64_t offset;      /* absolute offset in the file */
    uint64_t size_bytes;
} KSerTensorEntry;

typedef struct {
    int valid;
    char model_name[64];
    uint32_t vocab_size;
    uint32_t dim;
    uint32_t n_layers;
    uint8_t dtype;
    uint64_t n_params;
    uint64_t file_size;
} KSerInfo;

typedef struct KSerWriter KSerWriter;
typedef struct KSerReader KSerReader;
typedef int (*KSerVocabCallback)(uint32_t id, const char *token, uint16_t len, void *userdata);

/* Writer (reference kser_write.c): the file is written to "<path>.tmp" and
 * renamed to path when kser_writer_free() follows a successful finalize. */
KSerWriter *kser_writer_create(const char *path, const KSerConfig *cfg);
int kser_writer_add_vocab(KSerWriter *w, uint32_t id, const char *token, uint16_t len);
int kser_writer_add_tensor(KSerWriter *w, const char *name, const void *data, const uint32_t shape[4],
                           KSerDtype src_dtype, KSerDtype storage_dtype);
int kser_writer_finalize(KSerWriter *w);
void kser_writer_free(KSerWriter *w);

/* Reader (reference kser_read.c).  The SHA-256 is checked at open on every
 * path (the reference checks it only when mmap fails, so its
 * kser_reader_is_valid() is 0 on POSIX): kser_reader_is_valid() = 1 when the
 * stored checksum matches. */
KSerReader *kser_reader_open(const char *path);
const KSerConfig *kser_reader_config(KSerReader *r);
int kser_reader_is_valid(KSerReader *r);
int kser_reader_load_vocab(KSerReader *r, KSerVocabCallback cb, void *userdata);
/* malloc'd float32 copy (dequantized) of the named tensor, or NULL; free() it. */
float *kser_reader_load_tensor(KSerReader *r, const char *name);
uint64_t kser_reader_count_tensors(KSerReader *r);
const KSerTensorEntry *kser_reader_get_tensor_info(KSerReader *r, uint64_t idx);
void kser_reader_close(KSerReader *r);

KSerInfo kser_file_info(const char *path);

/* Conversions of the format (reference kser_quantize.c): fp16 by mantissa
 * truncation, bf16 by round-to-nearest-even, int8 as per-tensor min / range
 * (an 8-byte scale, zero-point header then n bytes). */
int kser_quantize(const float *src, void *dst, uint64_t n, KSerDtype dtype);
int kser_dequantize(const void *src, float *dst, uint64_t n, KSerDtype dtype);
size_t kser_dtype_size(KSerDtype dtype);

/* FIPS 180-4 SHA-256. */
void kser_sha256(const uint8_t *data, size_t len, uint8_t hash[32]);

#ifdef __cplusplus
}
#endif
#endif
