/*
 * Plain-C restatement of the elastic sparse index / causal-mask generator.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the device pattern kernel at sizes
 * where the numpy restatement (oracle/pattern.py) is too slow or too large.
 * Nothing in the shipped library links this file.
 *
 * Follows elastic_sparse_attention.py:470-535 (_create_elastic_sparse_indices).
 * Every step is one float32 operation with its own rounding, as torch does it
 * on the CPU; build with -ffp-contract=off so that no multiply-add is fused.
 * rintf() rounds half to even in the default rounding mode, like Tensor.round.
 */
#include <math.h>
#include <stdlib.h>
#include <stdint.h>
#include <string.h>

typedef struct {
    int w;
    float a_f32;        /* f32(alpha)                              :489 */
    float c_f32;        /* f32(w * (1 - alpha)), product in double  :496 */
} esa_oracle_layer;

static esa_oracle_layer make_layer(int w, int layer_idx, int num_hidden_layers) {
    esa_oracle_layer p;
    int denominator = num_hidden_layers > 1 ? num_hidden_layers - 1 : 1;   /* :488 */
    double a = (double)layer_idx / (double)denominator;                    /* :489 */
    p.w = w;
    p.a_f32 = (float)a;
    p.c_f32 = (float)((double)w * (1.0 - a));
    return p;
}

/* start (st) and spacing (sp) of one query row, :482-499 */
static void row_params(const esa_oracle_layer* p, int64_t pos, int64_t* st, float* sp) {
    int64_t end = pos > (int64_t)(p->w - 1) ? pos : (int64_t)(p->w - 1);   /* :483 */
    float E = (float)(end + 1);                                             /* :495 */
    volatile float prod = E * p->a_f32;
    float pd = p->c_f32 + prod;                                             /* :496 */
    float s = rintf(E - pd);                                                /* :497 */
    if (s < 0.0f) s = 0.0f;
    *st = (int64_t)s;
    *sp = (float)(end + 1 - *st) / (float)p->w;                             /* :498-499 */
}

/*
 * idx/mask [H, n, w] int64 for query rows positions[0..n) (or 0..n when
 * positions is NULL).  Masked slots get index 0, as the reference does.
 */
void esa_oracle_pattern(int num_heads, int64_t n, const int64_t* positions, int w,
                        int layer_idx, int num_hidden_layers,
                        int64_t* idx_out, int64_t* mask_out) {
    esa_oracle_layer p = make_layer(w, layer_idx, num_hidden_layers);
    int64_t ov[4097];
    float tw[1024];
    int h, k;
    int64_t r;
    if (w > 4096 || num_heads > 1024) return;
    for (h = 0; h < num_heads; ++h)                                        /* :515-516 */
        tw[h] = num_heads > 1 ? (float)h / (float)(num_heads - 1) : 0.0f;
    for (r = 0; r < n; ++r) {
        int64_t pos = positions ? positions[r] : r;
        int64_t st;
        float sp;
        row_params(&p, pos, &st, &sp);
        for (k = 0; k <= w; ++k) {                                         /* :503-506 */
            volatile float m = (float)k * sp;
            ov[k] = st + (int64_t)rintf(m);
        }
        for (h = 0; h < num_heads; ++h) {
            float t = tw[h];
            float omt = 1.0f - t;
            int64_t* io = idx_out + ((int64_t)h * n + r) * w;
            int64_t* mo = mask_out + ((int64_t)h * n + r) * w;
            for (k = 0; k < w; ++k) {                                      /* :510-526 */
                volatile float x = (float)ov[k] * omt;
                volatile float y = (float)(ov[k + 1] - 1) * t;
                float v = x + y;
                int64_t id = (int64_t)rintf(v);
                int ok = id <= pos;                                        /* :532 */
                io[k] = ok ? id : 0;                                       /* :533 */
                mo[k] = ok;
            }
        }
    }
}

/*
 * Audit used by the tests: for every (head, slot), is the raw index
 * non-decreasing along query rows 0..n-1?  Returns the number of violations
 * (0 means the per-slot index columns are sorted, which the backward's
 * key-side enumeration relies on).  Also reports, through *max_step, the
 * largest increase of a raw index between consecutive rows.
 */
int64_t esa_oracle_audit(int num_heads, int64_t n, int w, int layer_idx,
                         int num_hidden_layers, int64_t* max_step) {
    esa_oracle_layer p = make_layer(w, layer_idx, num_hidden_layers);
    int64_t* prev;
    int64_t ov[4097];
    float tw[1024];
    int64_t bad = 0, mstep = 0, r;
    int h, k;
    if (w > 4096 || num_heads > 1024) return -1;
    prev = (int64_t*)malloc(sizeof(int64_t) * (size_t)num_heads * (size_t)w);
    if (!prev) return -1;
    for (h = 0; h < num_heads; ++h)
        tw[h] = num_heads > 1 ? (float)h / (float)(num_heads - 1) : 0.0f;
    for (r = 0; r < n; ++r) {
        int64_t st;
        float sp;
        row_params(&p, r, &st, &sp);
        for (k = 0; k <= w; ++k) {
            volatile float m = (float)k * sp;
            ov[k] = st + (int64_t)rintf(m);
        }
        for (h = 0; h < num_heads; ++h) {
            float t = tw[h];
            float omt = 1.0f - t;
            for (k = 0; k < w; ++k) {
                volatile float x = (float)ov[k] * omt;
                volatile float y = (float)(ov[k + 1] - 1) * t;
                int64_t id = (int64_t)rintf(x + y);
                if (r > 0) {
                    int64_t d = id - prev[h * w + k];
                    if (d < 0) ++bad;
                    if (d > mstep) mstep = d;
                }
                prev[h * w + k] = id;
            }
        }
    }
    free(prev);
    if (max_step) *max_step = mstep;
    return bad;
}
