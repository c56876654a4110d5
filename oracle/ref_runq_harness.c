/* Harness that compiles the reference's runq/runq.c unchanged (included from the reference tree with -DTESTING,
 * which drops its main(), runq.c:1142) and exports quantize(), the CPU matmul and forward() to ctypes.
 * TEST INFRASTRUCTURE ONLY: only the tests, smoke() and bench.py's CPU-baseline leg load it, as the checker.
 *
 * Built twice by oracle/Makefile:
 *   _ref/libref_runq.so       CPU build: matmul() is the plain C loop of runq.c:432-458.
 *   _ref/libref_runq_b200.so  -DFPGA build: matmul() calls fpga_matvec() (runq.c:461-474) from libmatvec_b200.so;
 *                             the CPU loop stays available as matmul_cpu().
 */
#define TESTING
#include "runq.c"

#ifdef FPGA
#define CPU_MATMUL matmul_cpu
#else
#define CPU_MATMUL matmul
#endif

void ref_runq_quantize(int8_t *q, float *s, float *x, int n, int gs) {
    QuantizedTensor t;
    memset(&t, 0, sizeof t);
    t.q = q;
    t.s = s;
    GS = gs;
    quantize(&t, x, n);
}

void ref_runq_matmul_cpu(float *out, const int8_t *wq, const float *ws, const int8_t *xq, const float *xs, int n,
                         int d, int gs) {
    QuantizedTensor x, w;
    memset(&x, 0, sizeof x);
    memset(&w, 0, sizeof w);
    x.q = (int8_t *)xq;
    x.s = (float *)xs;
    w.q = (int8_t *)wq;
    w.s = (float *)ws;
    GS = gs;
    CPU_MATMUL(out, &x, &w, n, d);
}

/* The CPU side of the isolated sweep for runq's int8 / fp32-scale matvec: `reps` back-to-back calls of runq.c's
 * CPU matmul, call r reading weight copy r % copies (wq + c * wstride values, ws + c * sstride scales). Returns
 * the wall-clock seconds of all calls. */
double ref_runq_time_matmul_cpu(float *out, const int8_t *wq, const float *ws, size_t wstride, size_t sstride,
                                int copies, const int8_t *xq, const float *xs, int n, int d, int gs, int reps) {
    QuantizedTensor x, w;
    memset(&x, 0, sizeof x);
    memset(&w, 0, sizeof w);
    x.q = (int8_t *)xq;
    x.s = (float *)xs;
    GS = gs;
    struct timespec t0, t1;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for (int r = 0; r < reps; r++) {
        const size_t c = (size_t)(r % copies);
        w.q = (int8_t *)wq + c * wstride;
        w.s = (float *)ws + c * sstride;
        CPU_MATMUL(out, &x, &w, n, d);
    }
    clock_gettime(CLOCK_MONOTONIC, &t1);
    return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}

static Transformer model;
static int model_open;

int ref_runq_open(const char *path) {
    if (model_open) return -1;
    build_transformer(&model, (char *)path);
    model_open = 1;
    return 0;
}

int ref_runq_config(int *out) {
    if (!model_open) return -1;
    const Config *c = &model.config;
    out[0] = c->dim; out[1] = c->hidden_dim; out[2] = c->n_layers; out[3] = c->n_heads; out[4] = c->n_kv_heads;
    out[5] = c->vocab_size; out[6] = c->seq_len; out[7] = GS;
    return 0;
}

/* Logits (vocab_size floats) of `token` at position `pos`; positions must be fed in order from 0. */
const float *ref_runq_forward(int token, int pos) { return forward(&model, token, pos); }

int ref_runq_argmax(float *logits, int n) { return sample_argmax(logits, n); }

void ref_runq_close(void) {
    if (model_open) free_transformer(&model);
    model_open = 0;
}
