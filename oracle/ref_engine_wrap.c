/* ref_engine_wrap.c -- builds the REFERENCE's own engine C (qwen_engine.c or
 * gpt2_engine.c, selected by -DREF_ENGINE_SRC and -DREF_QWEN / -DREF_GPT2)
 * unmodified into a shared library under oracle/_ref/, so tests can pin the
 * oracle restatement against the reference's cpu_forward / cpu_gemv(_h).
 *
 * TEST INFRASTRUCTURE ONLY.  The driver-API calls the engine declares are
 * stubbed to fail: only the CPU golden-model functions are ever called.
 * The engine file is #included, so its static functions are reachable from
 * the small exported wrappers at the end of this translation unit.
 */
#define main ref_engine_main
#include REF_ENGINE_SRC
#undef main

/* ---- driver-API stubs (never reached by the wrappers below) ---- */
CUresult cuInit(unsigned int f) { (void)f; return 100; }
CUresult cuDeviceGet(CUdevice *d, int o) { (void)d; (void)o; return 100; }
CUresult cuCtxCreate_v2(CUcontext *c, unsigned f, CUdevice d) { (void)c; (void)f; (void)d; return 100; }
CUresult cuModuleLoadData(CUmodule *m, const void *i) { (void)m; (void)i; return 100; }
CUresult cuModuleGetFunction(CUfunction *f, CUmodule m, const char *n) { (void)f; (void)m; (void)n; return 100; }
CUresult cuMemAlloc_v2(CUdeviceptr *p, size_t b) { (void)p; (void)b; return 100; }
CUresult cuMemcpyHtoD_v2(CUdeviceptr d, const void *s, size_t b) { (void)d; (void)s; (void)b; return 100; }
CUresult cuMemcpyDtoH_v2(void *d, CUdeviceptr s, size_t b) { (void)d; (void)s; (void)b; return 100; }
CUresult cuMemcpyDtoD_v2(CUdeviceptr d, CUdeviceptr s, size_t b) { (void)d; (void)s; (void)b; return 100; }
CUresult cuLaunchKernel(CUfunction f, unsigned a, unsigned b, unsigned c, unsigned d, unsigned e,
                        unsigned g, unsigned h, CUstream s, void **p, void **x) {
    (void)f; (void)a; (void)b; (void)c; (void)d; (void)e; (void)g; (void)h; (void)s; (void)p; (void)x;
    return 100;
}
CUresult cuCtxSynchronize(void) { return 100; }
CUresult cuGetErrorString(CUresult r, const char **s) { (void)r; if (s) *s = "stub"; return 0; }

/* ---- exported wrappers ---- */
int ref_argmax_any(const float *v, int n) { return argmax(v, n); }
#ifdef REF_QWEN
static float *wrap_logits;
int ref_qwen_load(const char *path) {
    load_weights(path);                       /* exits on a bad file, as the reference does */
    kc_h = calloc((size_t)NL * CTX * KVD, 4);
    vc_h = calloc((size_t)NL * CTX * KVD, 4);
    ref_logits = malloc((size_t)V * 4);
    wrap_logits = ref_logits;
    return 0;
}
void ref_qwen_reset(void) {
    memset(kc_h, 0, (size_t)NL * CTX * KVD * 4);
    memset(vc_h, 0, (size_t)NL * CTX * KVD * 4);
}
void ref_qwen_forward(int token, int pos, int want_logits, float *logits_out) {
    cpu_forward(token, pos, want_logits, NULL);
    if (want_logits && logits_out) memcpy(logits_out, wrap_logits, (size_t)V * 4);
}
void ref_qwen_residual(float *out) { memcpy(out, r_x, sizeof(r_x)); }
void ref_gemv_h(const unsigned short *W, const float *x, const unsigned short *bias, float *y,
                int K, int N) {
    cpu_gemv_h(W, x, bias, y, K, N);
}
void ref_rms(const float *x, const unsigned short *w, float *y, int n) { cpu_rms(x, w, y, n); }
float ref_h2f(unsigned short h) { return h2f(h); }
int ref_argmax(const float *v, int n) { return argmax(v, n); }
/* sampler (qwen_engine.c:375-399) with the engine's own xorshift state */
void ref_sampler_seed(unsigned int s) { rng_state = s; }
int ref_sample_token(const float *logits, const int *ctx, int ctx_len) {
    return sample_token(logits, ctx, ctx_len);
}
#endif

#ifdef REF_GPT2
int ref_gpt2_load(const char *path) {
    load_weights(path);
    kc_h = calloc((size_t)NL * CTX * C, 4);
    vc_h = calloc((size_t)NL * CTX * C, 4);
    return 0;
}
void ref_gpt2_reset(void) {
    memset(kc_h, 0, (size_t)NL * CTX * C * 4);
    memset(vc_h, 0, (size_t)NL * CTX * C * 4);
}
void ref_gpt2_forward(int token, int pos, int want_logits, float *logits_out) {
    cpu_forward(token, pos, want_logits, NULL);
    if (want_logits && logits_out) memcpy(logits_out, ref_logits, (size_t)V * 4);
}
void ref_gpt2_residual(float *out) { memcpy(out, r_x, sizeof(r_x)); }
void ref_gemv(const float *W, const float *x, const float *bias, float *y, int K, int N) {
    cpu_gemv(W, x, bias, y, K, N);
}
void ref_ln(const float *x, const float *w, const float *b, float *y) { cpu_ln(x, w, b, y); }
#endif
