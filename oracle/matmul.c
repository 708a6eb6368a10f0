/*
 * matmul.c -- restatement of src/matmul.rs (oracle, test-only).
 *
 * The x86-64 build of the reference takes the scalar branches (`cfg(not(target_arch =
 * "aarch64"))`), so these are the functions restated: dot_product_scalar (:284-287),
 * dot_product_bf16_scalar (:289-295), dot_product_int8_scalar (:297-317) and dot_product_int4
 * (:149-173, the only int4 kernel on every architecture).  `Iterator::sum` for f32 folds from
 * -0.0 (Rust >= 1.82, required by the crate's edition 2024) left to right; the int4 loop starts
 * its accumulator at +0.0.  The two only differ for empty rows.
 */
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "pyxis_oracle.h"

static inline float bf16_bits_to_f32(uint16_t b) {
    uint32_t bits = (uint32_t)b << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* src/matmul.rs:284-287 */
float oracle_dot_f32(const float *a, const float *b, size_t len) {
    float sum = -0.0f;
    for (size_t i = 0; i < len; ++i) sum += a[i] * b[i];
    return sum;
}

/* src/matmul.rs:289-295 */
float oracle_dot_bf16(const float *a, const uint16_t *b, size_t len) {
    float sum = -0.0f;
    for (size_t i = 0; i < len; ++i) sum += a[i] * bf16_bits_to_f32(b[i]);
    return sum;
}

/* src/matmul.rs:297-317: input * quantized[g] as f32 * scales[g / block_size] */
float oracle_dot_int8(const float *x, const int8_t *q, const float *scales, size_t block_size,
                      size_t offset, size_t len) {
    float sum = -0.0f;
    for (size_t i = 0; i < len; ++i) {
        size_t g = offset + i;
        float t = x[i] * (float)q[g];
        t = t * scales[g / block_size];
        sum += t;
    }
    return sum;
}

/* src/matmul.rs:149-173: sum += *input_value * (nibble as f32 - 8.0) * scale */
float oracle_dot_int4(const float *x, const uint8_t *packed, const float *scales,
                      size_t block_size, size_t offset, size_t len) {
    float sum = 0.0f;
    for (size_t i = 0; i < len; ++i) {
        size_t g = offset + i;
        uint8_t byte = packed[g / 2];
        uint8_t nib = (g % 2 == 0) ? (byte & 0x0f) : ((byte >> 4) & 0x0f);
        float t = x[i] * ((float)nib - 8.0f);
        t = t * scales[g / block_size];
        sum += t;
    }
    return sum;
}

int oracle_num_cpus(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

typedef struct {
    const float *X;
    size_t M;
    int kind;
    const void *data;
    const float *scales;
    size_t block_size, out_features, in_features;
    float *Y;
    atomic_size_t next; /* dynamic chunking, like Rayon's work stealing over rows */
} mm_job;

enum { MM_CHUNK = 16 };

static void mm_rows(mm_job *j, size_t m, size_t r0, size_t r1) {
    const float *x = j->X + m * j->in_features;
    float *y = j->Y + m * j->out_features;
    size_t K = j->in_features;
    for (size_t r = r0; r < r1; ++r) {
        size_t row_start = r * K; /* src/matmul.rs:70 */
        switch (j->kind) {
        case ORACLE_F32: y[r] = oracle_dot_f32(x, (const float *)j->data + row_start, K); break;
        case ORACLE_BF16: y[r] = oracle_dot_bf16(x, (const uint16_t *)j->data + row_start, K); break;
        case ORACLE_INT8:
            y[r] = oracle_dot_int8(x, (const int8_t *)j->data, j->scales, j->block_size, row_start, K);
            break;
        case ORACLE_INT4:
            y[r] = oracle_dot_int4(x, (const uint8_t *)j->data, j->scales, j->block_size, row_start, K);
            break;
        }
    }
}

static void *mm_worker(void *arg) {
    mm_job *j = (mm_job *)arg;
    size_t rows = j->out_features;
    size_t chunks_per_m = (rows + MM_CHUNK - 1) / MM_CHUNK;
    size_t total = chunks_per_m * j->M;
    for (;;) {
        size_t c = atomic_fetch_add(&j->next, 1);
        if (c >= total) break;
        size_t m = c / chunks_per_m, r0 = (c % chunks_per_m) * MM_CHUNK;
        size_t r1 = r0 + MM_CHUNK < rows ? r0 + MM_CHUNK : rows;
        mm_rows(j, m, r0, r1);
    }
    return NULL;
}

/* Shape checks of src/matmul.rs:27-50 for the arms this oracle handles. */
static int mm_check(int kind, size_t block_size, size_t out_features, size_t in_features) {
    if (kind < ORACLE_F32 || kind > ORACLE_INT4) return -1;
    if ((kind == ORACLE_INT8 || kind == ORACLE_INT4) && block_size == 0) return -1;
    (void)out_features;
    (void)in_features;
    return 0;
}

int oracle_matmul_batch(const float *X, size_t M, int kind, const void *data, const float *scales,
                        size_t block_size, size_t out_features, size_t in_features, float *Y,
                        int nthreads) {
    if (mm_check(kind, block_size, out_features, in_features)) return -1;
    if (out_features == 0 || M == 0) return 0;
    mm_job j = {X, M, kind, data, scales, block_size, out_features, in_features, Y, 0};
    atomic_init(&j.next, 0);
    int nt = nthreads > 0 ? nthreads : oracle_num_cpus();
    size_t work = ((out_features + MM_CHUNK - 1) / MM_CHUNK) * M;
    if ((size_t)nt > work) nt = (int)work;
    if (nt <= 1) {
        mm_worker(&j);
        return 0;
    }
    pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nt);
    if (!th) return -1;
    int started = 0;
    for (int t = 1; t < nt; ++t)
        if (pthread_create(&th[t], NULL, mm_worker, &j) == 0) ++started;
        else th[t] = 0;
    mm_worker(&j);
    for (int t = 1; t < nt; ++t)
        if (th[t]) pthread_join(th[t], NULL);
    free(th);
    (void)started;
    return 0;
}

int oracle_matmul(const float *x, int kind, const void *data, const float *scales,
                  size_t block_size, size_t out_features, size_t in_features, float *y,
                  int nthreads) {
    return oracle_matmul_batch(x, 1, kind, data, scales, block_size, out_features, in_features, y,
                               nthreads);
}

/* src/output_head.rs:30-44 */
size_t oracle_argmax(const float *values, size_t n) {
    size_t max_idx = 0;
    float max_value = values[0];
    for (size_t i = 1; i < n; ++i)
        if (values[i] > max_value) {
            max_idx = i;
            max_value = values[i];
        }
    return max_idx;
}
