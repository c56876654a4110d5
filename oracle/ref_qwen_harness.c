/* Harness that compiles the reference's qwen/qwen.c unchanged (included from the reference tree, never copied)
 * and exports its quantize(), matmul_cpu(), f16() and forward() to ctypes. TEST INFRASTRUCTURE ONLY: only the
 * tests, smoke() and bench.py's CPU-baseline leg load it, as the checker.
 *
 * Built twice by oracle/Makefile:
 *   _ref/libref_qwen.so       CPU build: forward() runs every matmul through matmul_cpu (qwen.c:407-457).
 *   _ref/libref_qwen_b200.so  -DFPGA build: forward() calls fpga_matvec4() (qwen.c:459-473), which resolves to
 *                             libmatvec_b200.so. The host code is the reference's, byte for byte.
 */
#define main qwen_reference_main
#include "qwen.c"
#undef main

void ref_qwen_quantize(int8_t *q, float *s, const float *x, int n) { quantize(q, s, x, n); }

float ref_qwen_f16(uint16_t h) { return f16(h); }

void ref_qwen_rmsnorm(float *o, const float *x, const float *w, int n, float eps) { rmsnorm(o, x, w, n, eps); }

void ref_qwen_matmul_cpu(float *out, const uint8_t *w, const uint16_t *s, const int8_t *xq, const float *xs, int n,
                         int d, int bits) {
    Matrix m;
    memset(&m, 0, sizeof m);
    m.w = w;
    m.s = s;
    m.n = n;
    m.d = d;
    m.bits = bits;
    matmul_cpu(out, &m, xq, xs);
}

/* The CPU side of the isolated matvec sweep: `reps` back-to-back calls of matmul_cpu (OpenMP over rows, as qwen.c
 * builds it), call r reading weight copy r % copies (w + c * wstride bytes, s + c * sstride scales) so that the
 * copies can be sized past the last-level cache. Returns the wall-clock seconds of all calls. */
double ref_qwen_time_matmul_cpu(float *out, const uint8_t *w, const uint16_t *s, size_t wstride, size_t sstride,
                                int copies, const int8_t *xq, const float *xs, int n, int d, int bits, int reps) {
    Matrix m;
    memset(&m, 0, sizeof m);
    m.n = n;
    m.d = d;
    m.bits = bits;
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (int r = 0; r < reps; r++) {
        const size_t c = (size_t)(r % copies);
        m.w = w + c * wstride;
        m.s = s + c * sstride;
        matmul_cpu(out, &m, xq, xs);
    }
    clock_gettime(CLOCK_MONOTONIC, &t1);
    return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}

static Transformer model;
static int model_open;

/* Loads a .qwb (and, in the -DFPGA build, opens the device and uploads the weights like qwen.c does). */
int ref_qwen_open(const char *path, int ctx) {
    if (model_open) return -1;
    build_transformer(&model, path, ctx);
    model_open = 1;
    return 0;
}

int ref_qwen_config(int *out) {
    if (!model_open) return -1;
    const Config *c = &model.c;
    out[0] = c->dim; out[1] = c->hidden_dim; out[2] = c->n_layers; out[3] = c->n_heads; out[4] = c->n_kv_heads;
    out[5] = c->vocab_size; out[6] = c->head_k; out[7] = model.ctx;
    return 0;
}

/* Head logits (head_k floats) of `token` at position `pos`; positions must be fed in order from 0. */
const float *ref_qwen_forward(int token, int pos) { return forward(&model, token, pos); }

const int32_t *ref_qwen_head_ids(void) { return model.w.head_ids; }

int ref_qwen_argmax(const float *logits, int n) { return sample_argmax(logits, n); }
