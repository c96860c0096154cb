/*
 * CPU ORACLE — test infrastructure only.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load this library; the product path in
 * spilltune_b200/ never does.
 *
 * Plain-C restatement of the reference's group-128 4-bit codec:
 *
 *   ram_vram_finetune/quantization/codecs.py
 *     encode()        :66-116  (int4-sym-g128 branch :93-105)
 *     unpack_codes()  :55-64   (int4: low nibble = even element, code-8)
 *     decode_into()   :158-170 (FP32 product code*scale, one RNE cast to BF16)
 *     validate_spec() :119-155 (reserved code 0, nonzero tail, scale checks)
 *
 * plus the NF4 codebook variant used by the benchmark configs ("NF4 group128":
 * same byte layout, 16-entry FP32 codebook, FP32 absmax per 128 elements).  The
 * NF4 variant has no reference implementation; its decode rule is the same
 * codebook-parametric rule bf16(fp32(lut[c]) * fp32(scale)).
 *
 * Everything is scalar and single threaded except oracle_decode_mt(), which
 * splits the flat range over pthreads for the timed CPU baseline.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <string.h>

#define GROUP 128

/* Round an IEEE binary32 to bfloat16, round-to-nearest-even (the rounding
 * torch's Tensor.copy_/to(bfloat16) applies).  NaN maps to a quiet NaN. */
uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u >> 16) | 0x0040u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return (uint16_t)(u >> 16);
}

float oracle_bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Reference int4 code table: code c in 0..15 decodes to c-8 (codecs.py:62). */
void oracle_int4_sym_lut(float lut[16]) {
    for (int c = 0; c < 16; ++c) lut[c] = (float)(c - 8);
}

/* decode_into (codecs.py:158-170), codebook-parametric.
 * payload: uint8[groups*64]; scales: float32[groups]; out: bf16 bits[numel]. */
void oracle_decode_g128(const uint8_t *payload, const float *scales, const float *lut,
                        int64_t numel, uint16_t *out) {
    for (int64_t i = 0; i < numel; ++i) {
        uint8_t byte = payload[i >> 1];
        int code = (i & 1) ? (byte >> 4) : (byte & 15);
        float v = lut[code] * scales[i / GROUP];
        out[i] = oracle_f32_to_bf16(v);
    }
}

struct decode_job {
    const uint8_t *payload; const float *scales; const float *lut;
    int64_t begin, end; uint16_t *out;
};

static void *decode_worker(void *p) {
    struct decode_job *j = (struct decode_job *)p;
    for (int64_t i = j->begin; i < j->end; ++i) {
        uint8_t byte = j->payload[i >> 1];
        int code = (i & 1) ? (byte >> 4) : (byte & 15);
        j->out[i] = oracle_f32_to_bf16(j->lut[code] * j->scales[i / GROUP]);
    }
    return 0;
}

/* Same as oracle_decode_g128, split over `threads` pthreads (group-aligned). */
void oracle_decode_mt(const uint8_t *payload, const float *scales, const float *lut,
                      int64_t numel, uint16_t *out, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    struct decode_job jobs[256];
    int64_t groups = (numel + GROUP - 1) / GROUP;
    int64_t per = (groups + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        int64_t b = (int64_t)t * per * GROUP, e = b + per * GROUP;
        if (b >= numel) break;
        if (e > numel) e = numel;
        jobs[t] = (struct decode_job){payload, scales, lut, b, e, out};
        pthread_create(&tid[t], 0, decode_worker, &jobs[t]);
        ++started;
    }
    for (int t = 0; t < started; ++t) pthread_join(tid[t], 0);
}

/* encode(mode='int4-sym-g128') (codecs.py:66-116): scale = absmax/7 with an
 * all-zero group mapped to 1.0; code = round_half_even(x/scale) clamped to
 * [-7,7], stored +8; two codes per byte, even element in the low nibble; the
 * ragged tail group is zero padded (so its padding codes are 8).
 * Returns 0, or -1 for a nonfinite input, -2 for a BF16-overflowing decode. */
int oracle_encode_int4_sym(const float *x, int64_t numel, uint8_t *payload, float *scales) {
    int64_t groups = (numel + GROUP - 1) / GROUP;
    for (int64_t g = 0; g < groups; ++g) {
        float chunk[GROUP];
        for (int i = 0; i < GROUP; ++i) {
            int64_t idx = g * GROUP + i;
            chunk[i] = idx < numel ? x[idx] : 0.0f;
            if (!isfinite(chunk[i])) return -1;
        }
        float amax = 0.0f;
        for (int i = 0; i < GROUP; ++i) { float a = fabsf(chunk[i]); if (a > amax) amax = a; }
        float scale = amax / 7.0f;
        if (scale == 0.0f) scale = 1.0f;
        scales[g] = scale;
        uint8_t q[GROUP];
        for (int i = 0; i < GROUP; ++i) {
            float n = chunk[i] / scale;
            if (n < -7.0f) n = -7.0f;
            if (n > 7.0f) n = 7.0f;
            q[i] = (uint8_t)((int)nearbyintf(n) + 8);
            float dec = (float)((int)q[i] - 8) * scale;
            uint16_t b = oracle_f32_to_bf16(dec);
            if ((b & 0x7f80u) == 0x7f80u) return -2;
        }
        for (int i = 0; i < GROUP / 2; ++i) payload[g * 64 + i] = (uint8_t)(q[2 * i] | (q[2 * i + 1] << 4));
    }
    return 0;
}

/* NF4 group-128 encoder (no reference counterpart): scale = absmax of the
 * group (1.0 for an all-zero group), code = index of the nearest codebook entry
 * to x/scale, ties to the lower index.  Tail padding encodes 0.0. */
int oracle_encode_nf4(const float *x, int64_t numel, const float *lut, uint8_t *payload, float *scales) {
    int64_t groups = (numel + GROUP - 1) / GROUP;
    for (int64_t g = 0; g < groups; ++g) {
        float chunk[GROUP];
        float amax = 0.0f;
        for (int i = 0; i < GROUP; ++i) {
            int64_t idx = g * GROUP + i;
            chunk[i] = idx < numel ? x[idx] : 0.0f;
            if (!isfinite(chunk[i])) return -1;
            float a = fabsf(chunk[i]);
            if (a > amax) amax = a;
        }
        float scale = amax == 0.0f ? 1.0f : amax;
        scales[g] = scale;
        uint8_t q[GROUP];
        for (int i = 0; i < GROUP; ++i) {
            float n = chunk[i] / scale;
            int best = 0;
            float bd = fabsf(n - lut[0]);
            for (int c = 1; c < 16; ++c) {
                float d = fabsf(n - lut[c]);
                if (d < bd) { bd = d; best = c; }
            }
            q[i] = (uint8_t)best;
        }
        for (int i = 0; i < GROUP / 2; ++i) payload[g * 64 + i] = (uint8_t)(q[2 * i] | (q[2 * i + 1] << 4));
    }
    return 0;
}

/* validate_spec int4 payload checks (codecs.py:143-150): returns 0 when valid,
 * 1 when a reserved code 0 appears inside the logical range, 2 when a padding
 * code past numel decodes to a nonzero value (code != 8), 3 for a nonpositive
 * or nonfinite scale, 4 for a decode that overflows BF16. */
int oracle_validate_int4_sym(const uint8_t *payload, const float *scales, int64_t numel) {
    const int64_t chunk_groups = 2048; /* VALIDATION_CHUNK_GROUPS, codecs.py:22 */
    int64_t groups = (numel + GROUP - 1) / GROUP;
    for (int64_t g = 0; g < groups; ++g)
        if (!(scales[g] > 0.0f) || !isfinite(scales[g])) return 3;
    for (int64_t g0 = 0; g0 < groups; g0 += chunk_groups) {
        int64_t g1 = g0 + chunk_groups < groups ? g0 + chunk_groups : groups;
        for (int64_t i = g0 * GROUP; i < g1 * GROUP; ++i) {
            uint8_t byte = payload[i >> 1];
            if (((i & 1) ? (byte >> 4) : (byte & 15)) == 0) return 1;
        }
        for (int64_t i = g0 * GROUP; i < g1 * GROUP; ++i) {
            uint8_t byte = payload[i >> 1];
            int code = (i & 1) ? (byte >> 4) : (byte & 15);
            if (i >= numel && code != 8) return 2;
        }
        for (int64_t i = g0 * GROUP; i < g1 * GROUP; ++i) {
            uint8_t byte = payload[i >> 1];
            int code = (i & 1) ? (byte >> 4) : (byte & 15);
            uint16_t b = oracle_f32_to_bf16((float)(code - 8) * scales[i / GROUP]);
            if ((b & 0x7f80u) == 0x7f80u) return 4;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------
 * bitsandbytes NF4 with double quantization, block 64 ("NF4-DQ64"), the
 * record the reference's Qwen3.5 NF4 path stages and multiplies
 * (ram_vram_finetune/quantization/nf4_backend.py:184-278 validates its
 * layout: packed uint8 [(numel+1)/2], absmax uint8 [ceil(numel/64)],
 * nested_absmax fp32 [ceil(blocks/256)], nested_quant_map fp32[256],
 * quant_map fp32[16], nested_offset >= 0).  bitsandbytes 0.50.2 is absent
 * here, so this is a restatement of its published format, PARITY UNPINNED:
 *   block absmax  a[b] = fp32(nested_map[absmax[b]] * nested_absmax[b / 256]) + offset
 *   element i     w[i] = bf16_rne(fp32(quant_map[code_i] * a[i / 64]))
 *   code_i        high nibble of packed[i / 2] for even i, low nibble for odd i.
 * ------------------------------------------------------------------------ */
#define DQ_BLOCK 64
#define DQ_NESTED 256

void oracle_nf4dq_absmax(const uint8_t *absmax_q, const float *nested_absmax, const float *nested_map,
                         float offset, int64_t blocks, float *out) {
    for (int64_t b = 0; b < blocks; ++b) {
        float v = nested_map[absmax_q[b]] * nested_absmax[b / DQ_NESTED];
        out[b] = v + offset;
    }
}

void oracle_nf4dq_decode(const uint8_t *packed, const float *absmax, const float *quant_map, int64_t numel,
                         uint16_t *out) {
    for (int64_t i = 0; i < numel; ++i) {
        uint8_t byte = packed[i >> 1];
        int code = (i & 1) ? (byte & 15) : (byte >> 4);
        out[i] = oracle_f32_to_bf16(quant_map[code] * absmax[i / DQ_BLOCK]);
    }
}

/* Nearest entry of a sorted-or-not table (ties to the lower index). */
static int nearest(const float *table, int n, float x) {
    int best = 0;
    float bd = fabsf(x - table[0]);
    for (int c = 1; c < n; ++c) {
        float d = fabsf(x - table[c]);
        if (d < bd) { bd = d; best = c; }
    }
    return best;
}

/* Test-fixture encoder of the same layout (no bitsandbytes available): block
 * absmax (1.0 for an all-zero block), NF4 code nearest to x/absmax; offset =
 * mean of the block absmaxes; (absmax - offset) quantized per 256 blocks to
 * the nearest nested_map entry of (absmax - offset) / max|absmax - offset|
 * (nested_absmax = that max, 1.0 when it is 0).  Returns the offset. */
float oracle_nf4dq_encode(const float *x, int64_t numel, const float *quant_map, const float *nested_map,
                          uint8_t *packed, uint8_t *absmax_q, float *nested_absmax, float *absmax_tmp) {
    int64_t blocks = (numel + DQ_BLOCK - 1) / DQ_BLOCK;
    double sum = 0.0;
    for (int64_t b = 0; b < blocks; ++b) {
        float amax = 0.0f;
        for (int i = 0; i < DQ_BLOCK; ++i) {
            int64_t idx = b * DQ_BLOCK + i;
            if (idx < numel && fabsf(x[idx]) > amax) amax = fabsf(x[idx]);
        }
        absmax_tmp[b] = amax == 0.0f ? 1.0f : amax;
        sum += absmax_tmp[b];
    }
    float offset = (float)(sum / (double)blocks);
    int64_t nb = (blocks + DQ_NESTED - 1) / DQ_NESTED;
    for (int64_t s = 0; s < nb; ++s) {
        float m = 0.0f;
        for (int64_t b = s * DQ_NESTED; b < blocks && b < (s + 1) * DQ_NESTED; ++b) {
            float d = fabsf(absmax_tmp[b] - offset);
            if (d > m) m = d;
        }
        nested_absmax[s] = m == 0.0f ? 1.0f : m;
        for (int64_t b = s * DQ_NESTED; b < blocks && b < (s + 1) * DQ_NESTED; ++b)
            absmax_q[b] = (uint8_t)nearest(nested_map, 256, (absmax_tmp[b] - offset) / nested_absmax[s]);
    }
    /* Codes against the absmax the decoder will reconstruct. */
    for (int64_t b = 0; b < blocks; ++b)
        absmax_tmp[b] = nested_map[absmax_q[b]] * nested_absmax[b / DQ_NESTED] + offset;
    if (numel > 0) memset(packed, 0, (size_t)((numel + 1) / 2));
    for (int64_t i = 0; i < numel; ++i) {
        float a = absmax_tmp[i / DQ_BLOCK];
        int code = nearest(quant_map, 16, a != 0.0f ? x[i] / a : 0.0f);
        if (i & 1) packed[i >> 1] |= (uint8_t)code;
        else packed[i >> 1] |= (uint8_t)(code << 4);
    }
    return offset;
}
