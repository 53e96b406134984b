/*
 * Serial float32 C restatement of the reference MatMulNBits algorithm.
 *
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and the
 * CPU-baseline legs of bench.py (via ctypes) as the checker or the timed CPU
 * baseline. The product library never links or calls it.
 *
 * Follows (paths relative to the xrGPU project root):
 *   kernels/_shared/extended/shaders/complex_kernel.glsl:80  nbitWeight
 *   kernels/_shared/extended/shaders/complex_kernel.glsl:83  packedMatmul (opcode 1025):
 *       for row: for col: sum=0; for k ascending: sum += A[row,k]*w(col,k);
 *       sum += bias[col]; store converted to A's dtype.
 *   kernels/_shared/extended/shaders/complex_kernel.glsl:20  complexReadF (u8 read as float)
 *   kernels/_shared/shaders/half.glsl:4-45                    binary16 <-> binary32 storage
 *       conversion: exact widening; narrowing rounds to nearest even, finite
 *       overflow goes to infinity, NaN stays NaN with a nonzero payload.
 * Packed uint8 zero points (extension) are unpacked low-first with row stride
 * ceil(blocks*bits/8), the order gatherQuant uses (complex_kernel.glsl:85).
 *
 * Build with -ffp-contract=off so every multiply and add rounds separately,
 * as the shader's float32 expressions are written.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { DT_F32 = 0, DT_F16 = 1, DT_U8 = 6, DT_NONE = -1 };

static float bits_to_float(uint32_t v) { float f; memcpy(&f, &v, 4); return f; }
static uint32_t float_to_bits(float f) { uint32_t v; memcpy(&v, &f, 4); return v; }

/* binary16 -> binary32, exact (every half value is a float value). */
float mmnb_oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    if (e == 31u) return bits_to_float(sign | 0x7f800000u | (m << 13));
    if (e == 0u) {
        /* subnormal: value = m * 2^-24, representable exactly in float */
        float v = (float)m * 5.9604644775390625e-8f;
        return sign ? -v : v;
    }
    return bits_to_float(sign | ((e + 112u) << 23) | (m << 13));
}

/* binary32 -> binary16, round to nearest even, overflow to infinity. */
uint16_t mmnb_oracle_f32_to_f16(float f) {
    uint32_t x = float_to_bits(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t e = (x >> 23) & 0xffu, m = x & 0x7fffffu;
    if (e == 0xffu) return (uint16_t)(m ? (sign | 0x7e00u | (m >> 13)) : (sign | 0x7c00u));
    int32_t he = (int32_t)e - 127 + 15;
    if (he >= 31) return (uint16_t)(sign | 0x7c00u);
    if (he <= 0) {
        if (he < -10) return (uint16_t)sign;
        uint32_t full = m | 0x800000u;
        uint32_t shift = (uint32_t)(14 - he);
        uint32_t q = full >> shift, rem = full & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)he << 10) | (m >> 13), rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q; /* carry may reach inf: correct */
    return (uint16_t)(sign | q);
}

void mmnb_oracle_f32_to_f16_array(const float* in, uint16_t* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = mmnb_oracle_f32_to_f16(in[i]);
}
void mmnb_oracle_f16_to_f32_array(const uint16_t* in, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = mmnb_oracle_f16_to_f32(in[i]);
}

typedef struct {
    const void* a; int a_dtype; int64_t rows, K, N;
    const uint8_t* b; const void* scales; const void* zp; int zp_dtype;
    const void* bias; int64_t bs, bits;
    void* y; float* w_out;
    int64_t col0, col1;
} job_t;

static float read_f(const void* p, int dtype, int64_t i) {
    if (dtype == DT_F32) return ((const float*)p)[i];
    if (dtype == DT_F16) return mmnb_oracle_f16_to_f32(((const uint16_t*)p)[i]);
    return (float)((const uint8_t*)p)[i];
}

/* nbitWeight (complex_kernel.glsl:80) for one (column, k). */
static float nbit_weight(const job_t* j, int64_t col, int64_t k) {
    int64_t blocks = (j->K + j->bs - 1) / j->bs;
    int64_t blob = (j->bs * j->bits + 7) / 8;
    int64_t element = k % j->bs, blk = k / j->bs;
    uint32_t shift = (uint32_t)((element * j->bits) % 8);
    uint32_t packed = j->b[(col * blocks + blk) * blob + (element * j->bits) / 8];
    uint32_t q = (packed >> shift) & ((1u << j->bits) - 1u);
    float z;
    if (j->zp_dtype == DT_NONE) {
        z = (float)(1u << (j->bits - 1));
    } else if (j->zp_dtype == DT_U8) {
        int64_t stride = (blocks * j->bits + 7) / 8;
        uint32_t byte = ((const uint8_t*)j->zp)[col * stride + (blk * j->bits) / 8];
        z = (float)((byte >> ((blk * j->bits) % 8)) & ((1u << j->bits) - 1u));
    } else {
        z = read_f(j->zp, j->zp_dtype, col * blocks + blk);
    }
    float s = read_f(j->scales, j->a_dtype, col * blocks + blk);
    float d = (float)q - z;
    return d * s;
}

static void* run_job(void* arg) {
    const job_t* j = (const job_t*)arg;
    if (j->w_out) {
        for (int64_t col = j->col0; col < j->col1; ++col)
            for (int64_t k = 0; k < j->K; ++k) j->w_out[col * j->K + k] = nbit_weight(j, col, k);
        return NULL;
    }
    for (int64_t row = 0; row < j->rows; ++row) {
        for (int64_t col = j->col0; col < j->col1; ++col) {
            float sum = 0.0f;
            for (int64_t k = 0; k < j->K; ++k) {
                float a = read_f(j->a, j->a_dtype, row * j->K + k);
                float w = nbit_weight(j, col, k);
                float p = a * w;
                sum = sum + p;
            }
            if (j->bias) sum = sum + read_f(j->bias, j->a_dtype, col);
            int64_t o = row * j->N + col;
            if (j->a_dtype == DT_F32) ((float*)j->y)[o] = sum;
            else ((uint16_t*)j->y)[o] = mmnb_oracle_f32_to_f16(sum);
        }
    }
    return NULL;
}

static int run_threads(job_t base, int threads) {
    if (base.col1 < base.col0 || base.col0 < 0 || base.col1 > base.N) return 1;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    int64_t span = base.col1 - base.col0;
    if (threads > span) threads = span > 0 ? (int)span : 1;
    job_t jobs[256];
    pthread_t tids[256];
    for (int t = 0; t < threads; ++t) {
        jobs[t] = base;
        jobs[t].col0 = base.col0 + span * t / threads;
        jobs[t].col1 = base.col0 + span * (t + 1) / threads;
    }
    for (int t = 1; t < threads; ++t)
        if (pthread_create(&tids[t], NULL, run_job, &jobs[t]) != 0) return 2;
    run_job(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(tids[t], NULL);
    return 0;
}

/*
 * Y[row, col] for col in [col0, col1) of a [rows, N] output in A's dtype.
 * zp_dtype: -1 none, 0 float32, 1 float16, 6 packed uint8. Returns 0 on success.
 */
int mmnb_oracle_matmul(const void* a, int a_dtype, int64_t rows, int64_t K, int64_t N,
                       const uint8_t* b, const void* scales, const void* zp, int zp_dtype,
                       const void* bias, int64_t block_size, int64_t bits,
                       void* y, int64_t col0, int64_t col1, int threads) {
    if ((a_dtype != DT_F32 && a_dtype != DT_F16) || K <= 0 || N <= 0 || block_size <= 0) return 1;
    if (bits != 2 && bits != 4 && bits != 8) return 1;
    job_t j = {a, a_dtype, rows, K, N, b, scales, zp, zp_dtype, bias, block_size, bits, y, NULL, col0, col1};
    return run_threads(j, threads);
}

/* W[n, k] = nbitWeight(n, k) as float32 [N, K]. */
int mmnb_oracle_dequantize(int scale_dtype, int64_t K, int64_t N, const uint8_t* b,
                           const void* scales, const void* zp, int zp_dtype,
                           int64_t block_size, int64_t bits, float* w_out, int threads) {
    if (K <= 0 || N <= 0 || block_size <= 0 || (bits != 2 && bits != 4 && bits != 8)) return 1;
    job_t j = {NULL, scale_dtype, 0, K, N, b, scales, zp, zp_dtype, NULL, block_size, bits, NULL, w_out, 0, N};
    return run_threads(j, threads);
}
