/* cli_refpath.h -- the reference engines' own per-stage decode, for the
 * command-line hosts' --ptx, --debug and --selftest options.
 *
 * rp_forward is gpu_forward of the reference (qwen_engine.c:205-269,
 * gpt2_engine.c:174-264): one launch per stage, through the kernels of a
 * module image looked up by the reference's names and launched with the
 * reference's geometry, so `--ptx M` runs whatever module M the operator
 * passes (this package's lib/qwen.cubin / lib/gpt2.cubin, or one built from
 * the reference's own kernels).  With --debug it prints the reference's
 * layer-0 stage dumps at position 0 ("g.<tag> first4=... sum=...").
 *
 * rp_cpu_forward is the reference's serial CPU forward (qwen_engine.c:
 * 292-358, gpt2_engine.c:363-421) restated here, in the host, for
 * --selftest: GPU logits against it at the last selftested position, as the
 * reference's selftest does (qwen_engine.c:494-521, gpt2_engine.c:475-537),
 * with the "c.<tag>" dumps under --debug. */
#ifndef CLI_REFPATH_H
#define CLI_REFPATH_H

typedef struct refpath refpath;

/* model: SB_MODEL_QWEN or SB_MODEL_GPT2.  module_path NULL: this package's
 * built-in image of that model's kernels.  Reads the weight file itself.
 * Exits the process on any failure, as the reference's CHK does. */
refpath *rp_open(int model, const char *weights, const char *module_path, int ctx);
void rp_close(refpath *r);
/* GPU, per-stage (reference gpu_forward); logits (V floats) when want_logits */
void rp_forward(refpath *r, int token, int pos, int want_logits, float *logits, int debug);
/* CPU serial forward (reference cpu_forward); logits when want_logits */
void rp_cpu_forward(refpath *r, int token, int pos, int want_logits, float *logits, int debug);
/* buf (layers x C floats) receives the residual after each layer of every
 * later forward, GPU and CPU (the reference's divergence trace,
 * gpt2_engine.c:478-492); NULL stops it. */
void rp_set_trace(refpath *r, float *buf);
/* GPT-2: 1 = bias-fused gemv_warp_b launches (the reference's --fused) */
void rp_set_fused(refpath *r, int fused);
/* the module path actually loaded (for the banner) */
const char *rp_module_name(const refpath *r);

#endif
