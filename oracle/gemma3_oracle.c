/*
 * TEST INFRASTRUCTURE -- CPU restatement of the Vortex-RT Gemma 3 Q8_0 token
 * loop, used only as the checker of the CUDA path (tests/, smoke() and the
 * CPU-baseline leg of bench.py).  The product never links this file.
 *
 * What it restates, in the reference's operation order (file:line are in the
 * reference tree):
 *   - Q8_0 mat-vec as the shaders compute it: per-lane fp32 partial sums over
 *     blocks strided by the lane count, then a tree reduction
 *     (shaders/q8_matvec.comp:36-69); lanes = 0 selects the fp64 sequential
 *     mat-vec of the reference's FFN test (src/ffn_test_main.cpp:217-250)
 *   - gelu_tanh * up (shaders/gelu_mul.comp:17-31, src/gemma3.cpp:1440-1452)
 *   - argmax, ties -> lower index, NaN never wins (shaders/argmax.comp:30-107)
 *   - decode_token (src/gemma3.cpp:1462-1882): embedding row * sqrt(d)
 *     (1106-1136), rms_norm_into / rms_norm_inplace / rms_norm_heads_inplace
 *     with fp64 sums of squares (948-1104), NeoX RoPE from per-position
 *     tables (1309-1424), push-then-pop sliding-window KV (1590-1600),
 *     attention with fp64 dots and denominators (1609-1696), residuals,
 *     fused or unfused FFN (1713-1855), output norm, tied LM head + argmax or
 *     top-k (1138-1235)
 *   - generate_greedy_tokens (2080-2149)
 *   - the lane policy of Gemma3Model::q8_pipeline_for (655-671)
 * Generalised beyond the reference: any head_count_kv dividing head_count
 * (query head h reads KV head h / (H / KV)) and 64-bit tensor offsets.  With
 * head_count_kv == 1 the result is pinned bit for bit against the reference
 * itself (oracle/_ref); the GQA generalisation is exercised only here.
 *
 * Also holds the seeded synthetic-weight generator (same definition as
 * vortex-rt_b200/synth_gguf.py and the CUDA generator) so the 27B-shaped CPU
 * baseline can run without a 28.7 GB file.
 *
 * Compile with -ffp-contract=off: every product and sum rounds separately.
 */
#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ fp16 */

static float h2f(uint16_t h) { /* src/gguf.cpp:203-236 */
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 31u, m = h & 1023u, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else {
            int ex = -14;
            while ((m & 0x400u) == 0) { m <<= 1; --ex; }
            m &= 0x3ffu;
            bits = sign | ((uint32_t)(ex + 127) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e - 15u + 127u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* float -> half, round to nearest even (the synthetic generator's rule). */
static uint16_t f2h_rne(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | (ax > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) {
        if (ax < 0x33000000u) return (uint16_t)sign;
        uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u, shift = 126u - e;
        uint32_t mh = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (mh & 1u))) mh++;
        return (uint16_t)(sign | mh);
    }
    uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13), rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* ------------------------------------------------------- synthetic weights */

static uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    uint64_t z = x;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t fnv1a64(const char* s) {
    uint64_t h = 0xCBF29CE484222325ull;
    for (; *s; ++s) { h ^= (unsigned char)*s; h *= 0x100000001B3ull; }
    return h;
}

ORC_API uint64_t orc_stream_key(uint64_t seed, const char* name) {
    return splitmix64(seed ^ ((fnv1a64(name) + 1ull) * 0xD1B54A32D192ED03ull));
}

static int32_t irwin_hall(uint64_t key, uint64_t idx) {
    uint64_t h = splitmix64(key + idx);
    int64_t s = (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) + (int64_t)((h >> 32) & 0xFFFF) +
                (int64_t)(h >> 48);
    return (int32_t)(s - 131070);
}

/* Q8_0 bytes of rows [r0, r0+nr) of a synthetic N(0, std) [rows][cols] matrix. */
ORC_API void orc_synth_q8_rows(uint64_t key, uint32_t cols, uint64_t r0, uint64_t nr, double std_,
                               uint8_t* out) {
    const float mult = (float)(std_ / 37837.2265);
    float v[32];
    for (uint64_t r = 0; r < nr; ++r) {
        for (uint32_t b = 0; b < cols / 32u; ++b) {
            float amax = 0.0f;
            for (int k = 0; k < 32; ++k) {
                uint64_t idx = (r0 + r) * cols + (uint64_t)b * 32u + (uint64_t)k;
                v[k] = (float)irwin_hall(key, idx) * mult;
                float a = fabsf(v[k]);
                if (a > amax) amax = a;
            }
            float scale = amax == 0.0f ? 1.0f : amax / 127.0f;
            uint16_t hs = f2h_rne(scale);
            float dq = h2f(hs);
            uint8_t* blk = out + (r * (cols / 32u) + b) * 34u;
            blk[0] = (uint8_t)(hs & 0xff);
            blk[1] = (uint8_t)(hs >> 8);
            for (int k = 0; k < 32; ++k) {
                float q = rintf(v[k] / dq);
                if (q > 127.0f) q = 127.0f;
                if (q < -127.0f) q = -127.0f;
                blk[2 + k] = (uint8_t)(int8_t)q;
            }
        }
    }
}

ORC_API void orc_synth_norm(uint64_t key, uint32_t n, double std_, float* out) {
    const float mult = (float)(std_ / 37837.2265);
    for (uint32_t i = 0; i < n; ++i) out[i] = 1.0f + (float)irwin_hall(key, i) * mult;
}

/* ------------------------------------------------------------ thread pool */

typedef void (*range_fn)(void* ctx, uint64_t r0, uint64_t r1);
typedef struct { range_fn fn; void* ctx; uint64_t r0, r1; } range_job;

static void* range_entry(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->r0, j->r1);
    return NULL;
}

static void parallel_rows_min(int threads, uint64_t n, uint64_t min_per_thread, range_fn fn, void* ctx) {
    if (min_per_thread == 0) min_per_thread = 1;
    if ((uint64_t)threads > n / min_per_thread) threads = (int)(n / min_per_thread);
    if (threads <= 1) { fn(ctx, 0, n); return; }
    pthread_t tid[256];
    range_job jobs[256];
    if (threads > 256) threads = 256;
    for (int t = 0; t < threads; ++t) {
        jobs[t].fn = fn;
        jobs[t].ctx = ctx;
        jobs[t].r0 = n * (uint64_t)t / (uint64_t)threads;
        jobs[t].r1 = n * (uint64_t)(t + 1) / (uint64_t)threads;
        if (t > 0) pthread_create(&tid[t], NULL, range_entry, &jobs[t]);
    }
    range_entry(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
}

static void parallel_rows(int threads, uint64_t n, range_fn fn, void* ctx) {
    parallel_rows_min(threads, n, 16, fn, ctx);
}

/* ------------------------------------------------------------- Q8 mat-vec */

typedef struct {
    const uint8_t* w;
    uint32_t in, lanes;
    const float* x;
    float* y;
} mv_ctx;

static float shader_row(const uint8_t* row, uint32_t in, const float* x, uint32_t lanes) {
    float partial[64];
    uint32_t blocks = in / 32u;
    for (uint32_t lane = 0; lane < lanes; ++lane) {
        float sum = 0.0f;
        for (uint32_t b = lane; b < blocks; b += lanes) {
            const uint8_t* blk = row + (uint64_t)b * 34u;
            float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
            for (uint32_t k = 0; k < 32u; ++k) {
                float prod = d * (float)(int8_t)blk[2 + k];
                sum = sum + prod * x[b * 32u + k];
            }
        }
        partial[lane] = sum;
    }
    for (uint32_t stride = lanes / 2u; stride > 0u; stride >>= 1) {
        for (uint32_t lane = 0; lane < stride; ++lane) partial[lane] += partial[lane + stride];
    }
    return partial[0];
}

static float f64_row(const uint8_t* row, uint32_t in, const float* x) {
    double sum = 0.0;
    for (uint32_t b = 0; b < in / 32u; ++b) {
        const uint8_t* blk = row + (uint64_t)b * 34u;
        float d = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
        for (uint32_t k = 0; k < 32u; ++k) {
            float wv = d * (float)(int8_t)blk[2 + k];
            sum += (double)wv * (double)x[b * 32u + k];
        }
    }
    return (float)sum;
}

static void mv_range(void* p, uint64_t r0, uint64_t r1) {
    mv_ctx* c = (mv_ctx*)p;
    uint64_t row_bytes = (uint64_t)c->in / 32u * 34u;
    for (uint64_t r = r0; r < r1; ++r) {
        const uint8_t* row = c->w + r * row_bytes;
        c->y[r] = c->lanes ? shader_row(row, c->in, c->x, c->lanes) : f64_row(row, c->in, c->x);
    }
}

/* y[out] = W[out][in] x, W raw Q8_0 rows.  lanes in {8,16,32,64}; 0 = fp64 sequential. */
ORC_API void orc_q8_matvec(const uint8_t* w, const float* x, float* y, uint32_t in, uint32_t out,
                           uint32_t lanes, int threads) {
    mv_ctx c = {w, in, lanes, x, y};
    parallel_rows(threads, out, mv_range, &c);
}

static float gelu_tanh(float x) {
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    float x3 = x * x * x;
    return 0.5f * x * (1.0f + tanhf(k0 * (x + k1 * x3)));
}

ORC_API void orc_gelu_mul(float* gate, const float* up, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) gate[i] = gelu_tanh(gate[i]) * up[i];
}

ORC_API void orc_argmax(const float* v, uint32_t n, uint32_t* index, float* value) {
    float best = -INFINITY;
    uint32_t bi = 0xffffffffu;
    for (uint32_t i = 0; i < n; ++i) {
        float c = v[i];
        if (isnan(c)) continue;
        if (c > best || (c == best && i < bi)) { best = c; bi = i; }
    }
    *index = bi;
    *value = best;
}

/* --------------------------------------------------------------- GGUF read */

typedef struct {
    char name[96];
    uint32_t type, ndim;
    uint64_t dims[4];
    uint64_t offset;
} orc_tensor;

typedef struct {
    uint32_t ctx_len, d, L, ff, H, KV, hd, vd, vocab, window;
    float eps, theta_g, theta_l;
    uint64_t eos;
} orc_config;

typedef struct {
    float* keys;   /* [cap][KV*hd] ring (local) or linear (global) */
    float* values;
    uint32_t cap, count, start; /* deque state: entries start..start+count (mod cap) */
} orc_kv;

typedef struct orc_model {
    orc_config c;
    /* weights */
    uint8_t* map;
    size_t map_len;
    uint8_t* owned; /* synthetic models own their Q8 bytes */
    const uint8_t* data;
    orc_tensor* tensors;
    uint32_t n_tensors;
    const uint8_t *embd, **wq, **wk, **wv, **wo, **wg, **wu, **wd;
    float **n_attn, **n_q, **n_k, **n_post_attn, **n_ffn, **n_post_ffw, *n_out;
    float *rope_inv_local, *rope_inv_global;
    /* policy */
    uint32_t narrow_lanes;
    int force_lanes, fusion, threads;
    /* state */
    orc_kv* kv;
    uint32_t next_pos;
    float* trace; /* optional [L][d] per-layer hidden */
    char err[256];
} orc_model;

typedef struct { const uint8_t* p; const uint8_t* end; int bad; } rd;

static uint64_t rd_u(rd* r, int n) {
    uint64_t v = 0;
    if (r->p + n > r->end) { r->bad = 1; return 0; }
    memcpy(&v, r->p, (size_t)n);
    r->p += n;
    return v;
}

static void rd_str(rd* r, char* out, size_t cap) {
    uint64_t n = rd_u(r, 8);
    if (r->bad || r->p + n > r->end) { r->bad = 1; return; }
    if (out) {
        size_t m = n < cap - 1 ? (size_t)n : cap - 1;
        memcpy(out, r->p, m);
        out[m] = 0;
    }
    r->p += n;
}

static const int k_scalar_size[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};

static double rd_number(rd* r, uint32_t t, int* ok) {
    *ok = 1;
    switch (t) {
    case 0: return (double)(uint8_t)rd_u(r, 1);
    case 1: return (double)(int8_t)rd_u(r, 1);
    case 2: return (double)(uint16_t)rd_u(r, 2);
    case 3: return (double)(int16_t)rd_u(r, 2);
    case 4: return (double)(uint32_t)rd_u(r, 4);
    case 5: return (double)(int32_t)rd_u(r, 4);
    case 6: { uint32_t b = (uint32_t)rd_u(r, 4); float f; memcpy(&f, &b, 4); return f; }
    case 7: return (double)rd_u(r, 1);
    case 10: return (double)rd_u(r, 8);
    case 11: return (double)(int64_t)rd_u(r, 8);
    case 12: { uint64_t b = rd_u(r, 8); double f; memcpy(&f, &b, 8); return f; }
    default: *ok = 0; return 0;
    }
}

static void rd_skip_value(rd* r, uint32_t t, int depth) {
    if (depth > 8) { r->bad = 1; return; }
    if (t == 8) { rd_str(r, NULL, 0); return; }
    if (t == 9) {
        uint32_t et = (uint32_t)rd_u(r, 4);
        uint64_t n = rd_u(r, 8);
        if (et <= 12 && et != 8 && et != 9) {
            uint64_t bytes = n * (uint64_t)k_scalar_size[et];
            if (r->p + bytes > r->end) { r->bad = 1; return; }
            r->p += bytes;
            return;
        }
        for (uint64_t i = 0; i < n && !r->bad; ++i) rd_skip_value(r, et, depth + 1);
        return;
    }
    if (t > 12) { r->bad = 1; return; }
    r->p += k_scalar_size[t];
}

static orc_tensor* find_tensor(orc_model* m, const char* name) {
    for (uint32_t i = 0; i < m->n_tensors; ++i)
        if (strcmp(m->tensors[i].name, name) == 0) return &m->tensors[i];
    return NULL;
}

static int set_err(orc_model* m, const char* msg) {
    snprintf(m->err, sizeof m->err, "%s", msg);
    return -1;
}

static void build_rope_inv(float* inv, uint32_t hd, float theta) { /* gemma3.cpp:1309-1341 */
    for (uint32_t i = 0; i < hd / 2u; ++i) {
        float exponent = (2.0f * (float)i) / (float)hd;
        inv[i] = 1.0f / powf(theta, exponent);
    }
}

static int model_alloc_state(orc_model* m) {
    orc_config* c = &m->c;
    uint32_t L = c->L;
    m->wq = calloc(L, sizeof(void*)); m->wk = calloc(L, sizeof(void*)); m->wv = calloc(L, sizeof(void*));
    m->wo = calloc(L, sizeof(void*)); m->wg = calloc(L, sizeof(void*)); m->wu = calloc(L, sizeof(void*));
    m->wd = calloc(L, sizeof(void*));
    m->n_attn = calloc(L, sizeof(float*)); m->n_q = calloc(L, sizeof(float*)); m->n_k = calloc(L, sizeof(float*));
    m->n_post_attn = calloc(L, sizeof(float*)); m->n_ffn = calloc(L, sizeof(float*));
    m->n_post_ffw = calloc(L, sizeof(float*));
    m->kv = calloc(L, sizeof(orc_kv));
    m->rope_inv_local = malloc(sizeof(float) * c->hd / 2u);
    m->rope_inv_global = malloc(sizeof(float) * c->hd / 2u);
    build_rope_inv(m->rope_inv_local, c->hd, c->theta_l);
    build_rope_inv(m->rope_inv_global, c->hd, c->theta_g);
    return 0;
}

static int is_global(uint32_t layer) { return ((layer + 1u) % 6u) == 0u; }

static void set_policy(orc_model* m, uint32_t subgroup, uint32_t lane_override, int fusion) {
    /* gemma3.cpp:94-172 with a CPU device: fusion on only for subgroup 8. */
    m->fusion = fusion < 0 ? (subgroup == 8u) : fusion;
    m->force_lanes = lane_override != 0;
    uint32_t lanes = lane_override ? lane_override : (subgroup == 8 || subgroup == 16 || subgroup == 32 ? subgroup : 64u);
    m->narrow_lanes = lanes;
}

static uint32_t lanes_for(orc_model* m, uint32_t input_dim) { /* gemma3.cpp:655-671 */
    if (m->narrow_lanes != 64u && (m->force_lanes || input_dim <= 1024u)) return m->narrow_lanes;
    return 64u;
}

static int kv_alloc(orc_model* m, uint32_t max_positions) {
    orc_config* c = &m->c;
    size_t row = (size_t)c->KV * c->hd;
    for (uint32_t l = 0; l < c->L; ++l) {
        uint32_t cap = (!is_global(l) && c->window) ? c->window : max_positions;
        if (cap > max_positions) cap = max_positions;
        m->kv[l].cap = cap;
        m->kv[l].keys = malloc(sizeof(float) * row * cap);
        m->kv[l].values = malloc(sizeof(float) * row * cap);
        if (!m->kv[l].keys || !m->kv[l].values) return set_err(m, "oracle KV allocation failed");
    }
    return 0;
}

ORC_API void orc_close(orc_model* m);

ORC_API orc_model* orc_open(const char* path, uint32_t subgroup, uint32_t lane_override, int fusion,
                            int threads, uint32_t max_positions, char* err, size_t errlen) {
    orc_model* m = calloc(1, sizeof(orc_model));
    int fd = open(path, O_RDONLY);
    struct stat st;
    if (fd < 0 || fstat(fd, &st) != 0) {
        snprintf(err, errlen, "Failed to open GGUF file: %s", path);
        if (fd >= 0) close(fd);
        free(m);
        return NULL;
    }
    m->map_len = (size_t)st.st_size;
    m->map = mmap(NULL, m->map_len, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m->map == MAP_FAILED) { snprintf(err, errlen, "mmap failed"); free(m); return NULL; }
    rd r = {m->map, m->map + m->map_len, 0};
    uint32_t magic = (uint32_t)rd_u(&r, 4), version = (uint32_t)rd_u(&r, 4);
    uint64_t nt = rd_u(&r, 8), nkv = rd_u(&r, 8);
    if (magic != 0x46554747u || version < 2 || version > 3 || nt > 1000000 || nkv > 1000000) {
        snprintf(err, errlen, "Invalid GGUF header");
        orc_close(m);
        return NULL;
    }
    orc_config* c = &m->c;
    c->eps = 1e-6f; c->theta_g = 1e6f; c->theta_l = 1e4f; c->eos = 1;
    uint32_t alignment = 32;
    char key[256];
    for (uint64_t i = 0; i < nkv && !r.bad; ++i) {
        rd_str(&r, key, sizeof key);
        uint32_t t = (uint32_t)rd_u(&r, 4);
        if (t == 8 || t == 9) { rd_skip_value(&r, t, 0); continue; }
        int ok;
        double v = rd_number(&r, t, &ok);
        if (!ok) { r.bad = 1; break; }
        if (!strcmp(key, "gemma3.context_length")) c->ctx_len = (uint32_t)v;
        else if (!strcmp(key, "gemma3.embedding_length")) c->d = (uint32_t)v;
        else if (!strcmp(key, "gemma3.block_count")) c->L = (uint32_t)v;
        else if (!strcmp(key, "gemma3.feed_forward_length")) c->ff = (uint32_t)v;
        else if (!strcmp(key, "gemma3.attention.head_count")) c->H = (uint32_t)v;
        else if (!strcmp(key, "gemma3.attention.head_count_kv")) c->KV = (uint32_t)v;
        else if (!strcmp(key, "gemma3.attention.key_length")) c->hd = (uint32_t)v;
        else if (!strcmp(key, "gemma3.attention.value_length")) c->vd = (uint32_t)v;
        else if (!strcmp(key, "gemma3.attention.layer_norm_rms_epsilon")) c->eps = (float)v;
        else if (!strcmp(key, "gemma3.attention.sliding_window")) c->window = (uint32_t)v;
        else if (!strcmp(key, "gemma3.rope.freq_base")) c->theta_g = (float)v;
        else if (!strcmp(key, "tokenizer.ggml.eos_token_id")) c->eos = (uint64_t)v;
        else if (!strcmp(key, "general.alignment")) alignment = (uint32_t)v;
    }
    m->n_tensors = (uint32_t)nt;
    m->tensors = calloc(nt ? nt : 1, sizeof(orc_tensor));
    for (uint64_t i = 0; i < nt && !r.bad; ++i) {
        orc_tensor* t = &m->tensors[i];
        rd_str(&r, t->name, sizeof t->name);
        t->ndim = (uint32_t)rd_u(&r, 4);
        if (t->ndim == 0 || t->ndim > 4) { r.bad = 1; break; }
        for (uint32_t k = 0; k < t->ndim; ++k) t->dims[k] = rd_u(&r, 8);
        t->type = (uint32_t)rd_u(&r, 4);
        t->offset = rd_u(&r, 8);
    }
    if (r.bad) { snprintf(err, errlen, "Unexpected end of GGUF file"); orc_close(m); return NULL; }
    uint64_t pos = (uint64_t)(r.p - m->map);
    uint64_t data_off = (pos + alignment - 1) / alignment * alignment;
    m->data = m->map + data_off;
    orc_tensor* emb = find_tensor(m, "token_embd.weight");
    if (!emb || emb->type != 8 || emb->dims[0] != c->d) {
        snprintf(err, errlen, "Unsupported token_embd.weight layout");
        orc_close(m);
        return NULL;
    }
    c->vocab = (uint32_t)emb->dims[1];
    if (!c->d || !c->L || !c->ff || !c->H || !c->KV || !c->hd || c->H % c->KV || c->vd != c->hd) {
        snprintf(err, errlen, "Gemma 3 configuration is unsupported");
        orc_close(m);
        return NULL;
    }
    m->embd = m->data + emb->offset;
    model_alloc_state(m);
    char name[128];
#define Q8T(dst, suffix)                                                                       \
    do {                                                                                       \
        snprintf(name, sizeof name, "blk.%u." suffix, l);                                      \
        orc_tensor* t_ = find_tensor(m, name);                                                 \
        if (!t_ || t_->type != 8) { snprintf(err, errlen, "Missing Gemma 3 tensor: %s", name); \
                                    orc_close(m); return NULL; }                               \
        dst[l] = m->data + t_->offset;                                                         \
    } while (0)
#define F32T(dst, suffix)                                                                      \
    do {                                                                                       \
        snprintf(name, sizeof name, "blk.%u." suffix, l);                                      \
        orc_tensor* t_ = find_tensor(m, name);                                                 \
        if (!t_ || t_->type != 0) { snprintf(err, errlen, "Missing Gemma 3 tensor: %s", name); \
                                    orc_close(m); return NULL; }                               \
        dst[l] = (float*)(m->data + t_->offset);                                               \
    } while (0)
    for (uint32_t l = 0; l < c->L; ++l) {
        Q8T(m->wq, "attn_q.weight"); Q8T(m->wk, "attn_k.weight"); Q8T(m->wv, "attn_v.weight");
        Q8T(m->wo, "attn_output.weight"); Q8T(m->wg, "ffn_gate.weight"); Q8T(m->wu, "ffn_up.weight");
        Q8T(m->wd, "ffn_down.weight");
        F32T(m->n_attn, "attn_norm.weight"); F32T(m->n_q, "attn_q_norm.weight");
        F32T(m->n_k, "attn_k_norm.weight"); F32T(m->n_post_attn, "post_attention_norm.weight");
        F32T(m->n_ffn, "ffn_norm.weight"); F32T(m->n_post_ffw, "post_ffw_norm.weight");
    }
    orc_tensor* on = find_tensor(m, "output_norm.weight");
    if (!on) { snprintf(err, errlen, "Missing Gemma 3 tensor: output_norm.weight"); orc_close(m); return NULL; }
    m->n_out = (float*)(m->data + on->offset);
    set_policy(m, subgroup, lane_override, fusion);
    m->threads = threads;
    if (max_positions == 0 || max_positions > c->ctx_len) max_positions = c->ctx_len;
    if (kv_alloc(m, max_positions)) { snprintf(err, errlen, "%s", m->err); orc_close(m); return NULL; }
    return m;
}

typedef struct { uint64_t key; uint32_t cols; uint8_t* out; } gen_ctx;

static void gen_range(void* pp, uint64_t r0, uint64_t r1) {
    gen_ctx* q = (gen_ctx*)pp;
    orc_synth_q8_rows(q->key, q->cols, r0, r1 - r0, 0.02f, q->out + r0 * (q->cols / 32u) * 34u);
}

/* A synthetic model generated in memory with the shared seeded generator:
 * the same weights synth_gguf.write_gguf would write for (shape, seed). */
ORC_API orc_model* orc_open_synthetic(const uint32_t* shape /* d,L,H,KV,hd,ff,vocab,window,ctx */,
                                      float eps, float theta_g, uint64_t seed, uint32_t subgroup,
                                      uint32_t lane_override, int fusion, int threads,
                                      uint32_t max_positions) {
    orc_model* m = calloc(1, sizeof(orc_model));
    orc_config* c = &m->c;
    c->d = shape[0]; c->L = shape[1]; c->H = shape[2]; c->KV = shape[3]; c->hd = shape[4];
    c->vd = shape[4]; c->ff = shape[5]; c->vocab = shape[6]; c->window = shape[7]; c->ctx_len = shape[8];
    c->eps = eps; c->theta_g = theta_g; c->theta_l = 1e4f; c->eos = 1;
    model_alloc_state(m);
    uint64_t qw = (uint64_t)c->H * c->hd, kw = (uint64_t)c->KV * c->hd;
    uint64_t per_layer = (qw + 2 * kw) * (c->d / 32u) * 34u + qw / 32u * 34u * c->d +
                         2ull * c->ff * (c->d / 32u) * 34u + (uint64_t)c->d * (c->ff / 32u) * 34u;
    uint64_t total = (uint64_t)c->vocab * (c->d / 32u) * 34u + per_layer * c->L;
    uint64_t norms = ((uint64_t)c->d * 4u + 2u * c->hd) * c->L + c->d;
    m->owned = malloc(total + norms * 4u);
    if (!m->owned) { free(m); return NULL; }
    uint8_t* p = m->owned;
    char name[128];
    struct job { uint64_t key; uint32_t cols; uint64_t rows; uint8_t* out; } jobs[1 + 7 * 256];
    int nj = 0;
#define GEN(dst, nm, rows_, cols_)                                                               \
    do {                                                                                         \
        jobs[nj].key = orc_stream_key(seed, nm); jobs[nj].cols = (cols_); jobs[nj].rows = (rows_); \
        jobs[nj].out = p; dst = p; p += (uint64_t)(rows_) * ((cols_) / 32u) * 34u; nj++;        \
    } while (0)
    GEN(m->embd, "token_embd.weight", c->vocab, c->d);
    for (uint32_t l = 0; l < c->L && l < 256; ++l) {
        snprintf(name, sizeof name, "blk.%u.attn_q.weight", l); GEN(m->wq[l], name, qw, c->d);
        snprintf(name, sizeof name, "blk.%u.attn_k.weight", l); GEN(m->wk[l], name, kw, c->d);
        snprintf(name, sizeof name, "blk.%u.attn_v.weight", l); GEN(m->wv[l], name, kw, c->d);
        snprintf(name, sizeof name, "blk.%u.attn_output.weight", l); GEN(m->wo[l], name, c->d, qw);
        snprintf(name, sizeof name, "blk.%u.ffn_gate.weight", l); GEN(m->wg[l], name, c->ff, c->d);
        snprintf(name, sizeof name, "blk.%u.ffn_up.weight", l); GEN(m->wu[l], name, c->ff, c->d);
        snprintf(name, sizeof name, "blk.%u.ffn_down.weight", l); GEN(m->wd[l], name, c->d, c->ff);
    }
    float* fp = (float*)p;
#define NRM(dst, fmt, n)                                                 \
    do {                                                                 \
        snprintf(name, sizeof name, fmt, l);                             \
        orc_synth_norm(orc_stream_key(seed, name), (n), 0.1f, fp);       \
        dst = fp; fp += (n);                                             \
    } while (0)
    for (uint32_t l = 0; l < c->L; ++l) {
        NRM(m->n_attn[l], "blk.%u.attn_norm.weight", c->d);
        NRM(m->n_q[l], "blk.%u.attn_q_norm.weight", c->hd);
        NRM(m->n_k[l], "blk.%u.attn_k_norm.weight", c->hd);
        NRM(m->n_post_attn[l], "blk.%u.post_attention_norm.weight", c->d);
        NRM(m->n_ffn[l], "blk.%u.ffn_norm.weight", c->d);
        NRM(m->n_post_ffw[l], "blk.%u.post_ffw_norm.weight", c->d);
    }
    orc_synth_norm(orc_stream_key(seed, "output_norm.weight"), c->d, 0.1f, fp);
    m->n_out = fp;
    /* generate Q8 tensors row-parallel */
    for (int j = 0; j < nj; ++j) {
        gen_ctx g = {jobs[j].key, jobs[j].cols, jobs[j].out};
        parallel_rows(threads, jobs[j].rows, gen_range, &g);
    }
    set_policy(m, subgroup, lane_override, fusion);
    m->threads = threads;
    if (max_positions == 0 || max_positions > c->ctx_len) max_positions = c->ctx_len;
    if (kv_alloc(m, max_positions)) { orc_close(m); return NULL; }
    return m;
}

ORC_API void orc_close(orc_model* m) {
    if (!m) return;
    if (m->map && m->map != MAP_FAILED) munmap(m->map, m->map_len);
    free(m->owned);
    free(m->tensors);
    if (m->kv) {
        for (uint32_t l = 0; l < m->c.L; ++l) { free(m->kv[l].keys); free(m->kv[l].values); }
    }
    free(m->kv); free(m->wq); free(m->wk); free(m->wv); free(m->wo); free(m->wg); free(m->wu); free(m->wd);
    free(m->n_attn); free(m->n_q); free(m->n_k); free(m->n_post_attn); free(m->n_ffn); free(m->n_post_ffw);
    free(m->rope_inv_local); free(m->rope_inv_global);
    free(m);
}

ORC_API const char* orc_error(orc_model* m) { return m->err; }
ORC_API void orc_set_threads(orc_model* m, int t) { m->threads = t; }
ORC_API void orc_set_trace(orc_model* m, float* buf) { m->trace = buf; }
ORC_API void orc_config_get(orc_model* m, uint32_t* out, float* outf) {
    orc_config* c = &m->c;
    uint32_t v[10] = {c->ctx_len, c->d, c->L, c->ff, c->H, c->KV, c->hd, c->vd, c->vocab, c->window};
    memcpy(out, v, sizeof v);
    outf[0] = c->eps; outf[1] = c->theta_g; outf[2] = c->theta_l;
}
/* Raw Q8_0 bytes of a named weight (NULL if absent) for per-op parity tests. */
ORC_API const uint8_t* orc_weight(orc_model* m, const char* what, uint32_t layer) {
    if (!strcmp(what, "token_embd")) return m->embd;
    if (layer >= m->c.L) return NULL;
    if (!strcmp(what, "attn_q")) return m->wq[layer];
    if (!strcmp(what, "attn_k")) return m->wk[layer];
    if (!strcmp(what, "attn_v")) return m->wv[layer];
    if (!strcmp(what, "attn_output")) return m->wo[layer];
    if (!strcmp(what, "ffn_gate")) return m->wg[layer];
    if (!strcmp(what, "ffn_up")) return m->wu[layer];
    if (!strcmp(what, "ffn_down")) return m->wd[layer];
    return NULL;
}

ORC_API void orc_reset(orc_model* m) {
    for (uint32_t l = 0; l < m->c.L; ++l) { m->kv[l].count = 0; m->kv[l].start = 0; }
    m->next_pos = 0;
}

/* ------------------------------------------------------------ token step */

static void rms_into(const float* in, const float* w, float* out, uint32_t n, float eps) {
    double ss = 0.0;
    for (uint32_t i = 0; i < n; ++i) ss += (double)in[i] * (double)in[i];
    double mean = ss / (double)n;
    float scale = 1.0f / sqrtf((float)mean + eps);
    for (uint32_t i = 0; i < n; ++i) out[i] = in[i] * scale * w[i];
}

static void rms_inplace(float* v, const float* w, uint32_t n, float eps) {
    double ss = 0.0;
    for (uint32_t i = 0; i < n; ++i) ss += (double)v[i] * (double)v[i];
    double mean = ss / (double)n;
    float scale = 1.0f / sqrtf((float)mean + eps);
    for (uint32_t i = 0; i < n; ++i) v[i] *= scale * w[i];
}

static void rms_heads(float* v, uint32_t heads, uint32_t hd, const float* w, float eps) {
    for (uint32_t h = 0; h < heads; ++h) {
        float* x = v + (size_t)h * hd;
        double ss = 0.0;
        for (uint32_t i = 0; i < hd; ++i) ss += (double)x[i] * (double)x[i];
        float scale = 1.0f / sqrtf((float)(ss / (double)hd) + eps);
        for (uint32_t i = 0; i < hd; ++i) x[i] *= scale * w[i];
    }
}

static void rope(float* v, uint32_t heads, uint32_t hd, const float* cs, const float* sn) {
    uint32_t half = hd / 2u;
    for (uint32_t h = 0; h < heads; ++h) {
        float* x = v + (size_t)h * hd;
        for (uint32_t i = 0; i < half; ++i) {
            float a = x[i], b = x[half + i];
            x[i] = a * cs[i] - b * sn[i];
            x[half + i] = b * cs[i] + a * sn[i];
        }
    }
}

static void mv(orc_model* m, const uint8_t* w, const float* x, float* y, uint32_t in, uint32_t out,
               uint32_t lanes) {
    orc_q8_matvec(w, x, y, in, out, lanes, m->threads);
}

typedef struct {
    orc_model* m;
    uint32_t kvh_ratio;
    const float* q;
    orc_kv* kv;
    float* att;
} attn_ctx;

static void attn_heads(void* p, uint64_t h0, uint64_t h1) {
    attn_ctx* a = (attn_ctx*)p;
    orc_config* c = &a->m->c;
    const float scale_attn = 1.0f / sqrtf((float)c->hd);
    uint32_t n = a->kv->count, row = c->KV * c->hd;
    float* scores = malloc(sizeof(float) * (n ? n : 1));
    for (uint64_t h = h0; h < h1; ++h) {
        uint32_t g = (uint32_t)h / a->kvh_ratio;
        const float* qh = a->q + h * c->hd;
        float mx = -INFINITY;
        for (uint32_t t = 0; t < n; ++t) {
            uint32_t slot = (a->kv->start + t) % a->kv->cap;
            const float* k = a->kv->keys + (size_t)slot * row + (size_t)g * c->hd;
            double dot = 0.0;
            for (uint32_t d = 0; d < c->hd; ++d) dot += (double)qh[d] * (double)k[d];
            scores[t] = (float)dot * scale_attn;
            if (scores[t] > mx) mx = scores[t];
        }
        double den = 0.0;
        for (uint32_t t = 0; t < n; ++t) {
            float e = expf(scores[t] - mx);
            scores[t] = e;
            den += e;
        }
        float* out = a->att + h * c->vd;
        for (uint32_t d = 0; d < c->vd; ++d) out[d] = 0.0f;
        for (uint32_t t = 0; t < n; ++t) {
            float pr = (float)(scores[t] / den);
            uint32_t slot = (a->kv->start + t) % a->kv->cap;
            const float* v = a->kv->values + (size_t)slot * row + (size_t)g * c->hd;
            for (uint32_t d = 0; d < c->vd; ++d) out[d] += pr * v[d];
        }
    }
    free(scores);
}

/* One decode_token step.  Returns 0, writes hidden (d floats, after the
 * output norm) and the top-k (ids, logits) like Gemma3Model::top_logits. */
ORC_API int orc_decode(orc_model* m, uint32_t token, uint32_t position, uint32_t top_k, float* hidden_out,
                       uint32_t* ids, float* logits_out, uint32_t* n_top, float* full_logits) {
    orc_config* c = &m->c;
    if (position != m->next_pos) return set_err(m, "Gemma 3 decode positions must be contiguous");
    if (position >= c->ctx_len) return set_err(m, "Gemma 3 context length exceeded");
    if (token >= c->vocab) { orc_reset(m); return set_err(m, "Token id is outside Gemma 3 vocabulary"); }
    uint32_t d = c->d, qw = c->H * c->hd, kw = c->KV * c->hd, half = c->hd / 2u;
    float* hidden = malloc(sizeof(float) * d);
    float* xn = malloc(sizeof(float) * (d > c->ff ? d : c->ff));
    float* q = malloc(sizeof(float) * qw);
    float* k = malloc(sizeof(float) * kw);
    float* v = malloc(sizeof(float) * kw);
    float* att = malloc(sizeof(float) * qw);
    float* o = malloc(sizeof(float) * d);
    float* gate = malloc(sizeof(float) * c->ff);
    float* up = malloc(sizeof(float) * c->ff);
    float* lc = malloc(sizeof(float) * half), *ls = malloc(sizeof(float) * half);
    float* gcs = malloc(sizeof(float) * half), *gsn = malloc(sizeof(float) * half);
    int rc = 0;
    /* embedding: read_q8_0_row * sqrt(d) (gemma3.cpp:1106-1136, gguf.cpp:546-638) */
    const uint8_t* row = m->embd + (uint64_t)token * (d / 32u) * 34u;
    const float emb_scale = sqrtf((float)d);
    for (uint32_t b = 0; b < d / 32u; ++b) {
        const uint8_t* blk = row + (uint64_t)b * 34u;
        float s = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
        for (uint32_t j = 0; j < 32u; ++j) hidden[b * 32u + j] = s * (float)(int8_t)blk[2 + j];
    }
    for (uint32_t i = 0; i < d; ++i) hidden[i] *= emb_scale;
    const float pf = (float)position;
    for (uint32_t i = 0; i < half; ++i) {
        float al = pf * m->rope_inv_local[i], ag = pf * m->rope_inv_global[i];
        lc[i] = cosf(al); ls[i] = sinf(al);
        gcs[i] = cosf(ag); gsn[i] = sinf(ag);
    }
    uint32_t lanes_d = lanes_for(m, d);
    for (uint32_t l = 0; l < c->L; ++l) {
        rms_into(hidden, m->n_attn[l], xn, d, c->eps);
        mv(m, m->wq[l], xn, q, d, qw, lanes_d);
        mv(m, m->wk[l], xn, k, d, kw, lanes_d);
        mv(m, m->wv[l], xn, v, d, kw, lanes_d);
        rms_heads(q, c->H, c->hd, m->n_q[l], c->eps);
        rms_heads(k, c->KV, c->hd, m->n_k[l], c->eps);
        int glob = is_global(l);
        rope(q, c->H, c->hd, glob ? gcs : lc, glob ? gsn : ls);
        rope(k, c->KV, c->hd, glob ? gcs : lc, glob ? gsn : ls);
        orc_kv* kv = &m->kv[l];
        if (kv->count == kv->cap) { /* only a window-bounded ring may be full */
            if (glob || !c->window) { rc = set_err(m, "oracle KV capacity exceeded"); break; }
            kv->start = (kv->start + 1) % kv->cap;
            kv->count--;
        }
        uint32_t slot = (kv->start + kv->count) % kv->cap;
        memcpy(kv->keys + (size_t)slot * kw, k, sizeof(float) * kw);
        memcpy(kv->values + (size_t)slot * kw, v, sizeof(float) * kw);
        kv->count++;
        attn_ctx ac = {m, c->H / c->KV, q, kv, att};
        parallel_rows_min(kv->count * (uint64_t)c->hd >= 65536 ? m->threads : 1, c->H, 1, attn_heads, &ac);
        mv(m, m->wo[l], att, o, qw, d, lanes_for(m, qw));
        rms_inplace(o, m->n_post_attn[l], d, c->eps);
        for (uint32_t i = 0; i < d; ++i) o[i] += hidden[i];
        memcpy(hidden, o, sizeof(float) * d);
        rms_into(hidden, m->n_ffn[l], xn, d, c->eps);
        uint32_t lg = m->fusion ? lanes_d : lanes_d; /* gate/up: q8_pipeline_for(d) either way */
        mv(m, m->wg[l], xn, gate, d, c->ff, lg);
        mv(m, m->wu[l], xn, up, d, c->ff, lg);
        orc_gelu_mul(gate, up, c->ff);
        /* fused FFN keeps the d-wide pipeline for down; unfused picks by ff */
        mv(m, m->wd[l], gate, o, c->ff, d, m->fusion ? lanes_d : lanes_for(m, c->ff));
        rms_inplace(o, m->n_post_ffw[l], d, c->eps);
        for (uint32_t i = 0; i < d; ++i) o[i] += hidden[i];
        memcpy(hidden, o, sizeof(float) * d);
        for (uint32_t i = 0; i < d; ++i)
            if (!isfinite(hidden[i])) { rc = set_err(m, "Non-finite value after Gemma 3 block"); break; }
        if (rc) break;
        if (m->trace) memcpy(m->trace + (size_t)l * d, hidden, sizeof(float) * d);
    }
    if (!rc) {
        rms_inplace(hidden, m->n_out, d, c->eps);
        if (hidden_out) memcpy(hidden_out, hidden, sizeof(float) * d);
        uint32_t nt = 0;
        if (top_k > 0 || full_logits) {
            float* lg = full_logits ? full_logits : malloc(sizeof(float) * c->vocab);
            mv(m, m->embd, hidden, lg, d, c->vocab, lanes_d);
            if (top_k == 1) {
                uint32_t bi; float bv;
                orc_argmax(lg, c->vocab, &bi, &bv);
                if (bi >= c->vocab || !isfinite(bv)) rc = set_err(m, "GPU argmax produced invalid result");
                ids[0] = bi; logits_out[0] = bv; nt = 1;
            } else if (top_k > 1) {
                uint32_t kk = top_k < c->vocab ? top_k : c->vocab;
                /* selection by (logit desc, id asc); the reference's partial_sort
                 * leaves the order of equal logits unspecified */
                char* used = calloc(c->vocab, 1);
                for (uint32_t s = 0; s < kk; ++s) {
                    uint32_t bi = 0xffffffffu; float bv = -INFINITY;
                    for (uint32_t i = 0; i < c->vocab; ++i) {
                        if (used[i]) continue;
                        if (bi == 0xffffffffu || lg[i] > bv) { bi = i; bv = lg[i]; }
                    }
                    used[bi] = 1; ids[s] = bi; logits_out[s] = bv;
                }
                free(used);
                nt = kk;
            }
            if (!full_logits) free(lg);
        }
        if (n_top) *n_top = nt;
    }
    if (rc) orc_reset(m); else m->next_pos++;
    free(hidden); free(xn); free(q); free(k); free(v); free(att); free(o); free(gate); free(up);
    free(lc); free(ls); free(gcs); free(gsn);
    return rc;
}

/* generate_greedy_tokens (gemma3.cpp:2080-2149); margins[i] = top1 - top2 logit
 * of generated step i when `margins` is given (costs a full-logit pass). */
ORC_API int orc_generate(orc_model* m, const uint32_t* prompt, uint32_t n, uint32_t max_new, uint32_t* out,
                         uint32_t* out_n, float* margins) {
    orc_reset(m);
    *out_n = 0;
    if (max_new == 0) return 0;
    if (n == 0) return set_err(m, "Gemma 3 prompt produced no input tokens");
    uint32_t pos = 0, id = 0, nt = 0;
    float val = 0.0f;
    float* full = margins ? malloc(sizeof(float) * m->c.vocab) : NULL;
    int rc = 0;
    for (uint32_t i = 0; i < n && !rc; ++i) {
        int last = i + 1 == n;
        rc = orc_decode(m, prompt[i], pos++, last ? 1u : 0u, NULL, &id, &val, &nt, last ? full : NULL);
    }
    for (uint32_t i = 0; i < max_new && !rc; ++i) {
        if (i != 0) rc = orc_decode(m, id, pos++, 1u, NULL, &id, &val, &nt, full);
        if (rc) break;
        if (margins) {
            float second = -INFINITY;
            for (uint32_t j = 0; j < m->c.vocab; ++j)
                if (j != id && full[j] > second) second = full[j];
            margins[i] = val - second;
        }
        out[(*out_n)++] = id;
        if ((uint64_t)id == m->c.eos) break;
    }
    free(full);
    return rc;
}
