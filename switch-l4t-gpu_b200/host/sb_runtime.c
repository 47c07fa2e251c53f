/* sb_runtime.c -- context, module images and launches for libswitch_b200.
 *
 * The four sm_100a cubins are linked into the library (cubins.S) and loaded
 * with cuModuleLoadData into whichever context is current, exactly how the
 * reference's hosts load their PTX (gpu_workload.c:65-74); kernels are then
 * resolved by name with cuModuleGetFunction and launched with
 * cuLaunchKernel / cuLaunchKernelEx and void** parameter arrays. */
#define _GNU_SOURCE
#include <pthread.h>
#include <stdio.h>
#include <string.h>

#include "sb_internal.h"

extern const unsigned char sb_img_switch_gpu[], sb_img_switch_gpu_end[];
extern const unsigned char sb_img_gemv[], sb_img_gemv_end[];
extern const unsigned char sb_img_gpt2[], sb_img_gpt2_end[];
extern const unsigned char sb_img_qwen[], sb_img_qwen_end[];
extern const unsigned char sb_img_tc[], sb_img_tc_end[];

static const struct {
    const char *name;
    const unsigned char *lo, *hi;
} images[M_COUNT] = {
    {"switch_gpu", sb_img_switch_gpu, sb_img_switch_gpu_end},
    {"gemv", sb_img_gemv, sb_img_gemv_end},
    {"gpt2", sb_img_gpt2, sb_img_gpt2_end},
    {"qwen", sb_img_qwen, sb_img_qwen_end},
    {"tc", sb_img_tc, sb_img_tc_end},
};

static const struct {
    int mod;
    const char *name;
} fn_table[F_COUNT] = {
    [F_SGEMM_B200] = {M_SWITCH, "sgemm_b200"},
    [F_SGEMM_B200_DST] = {M_SWITCH, "sgemm_b200_dst"},
    [F_SGEMM_B200_STK] = {M_SWITCH, "sgemm_b200_stk"},
    [F_SGEMM_STK_FIXUP] = {M_SWITCH, "sgemm_stk_fixup"},
    [F_SGEMM_TMA] = {M_TC, "sgemm_tma"},
    [F_GEMM_HH_MMA8] = {M_QWEN, "gemm_hh_mma8"},
    [F_GEMM_HH_MMA16] = {M_QWEN, "gemm_hh_mma16"},
    [F_GEMM_HH_MMA8_W4] = {M_QWEN, "gemm_hh_mma8_w4"},
    [F_GEMM_HH_MMA16_W4] = {M_QWEN, "gemm_hh_mma16_w4"},
    [F_TOPK_PARTIAL] = {M_QWEN, "topk_partial"},
    [F_TOPK_MERGE] = {M_QWEN, "topk_merge"},
    [F_SGEMM_NAIVE] = {M_SWITCH, "sgemm_naive"},
    [F_MEMBW] = {M_SWITCH, "membw_read4"},
    [F_FMA_PEAK] = {M_SWITCH, "fma_peak"},
    [F_GEMV_F32_B200] = {M_GPT2, "gemv_f32_b200"},
    [F_GEMV_MULTI] = {M_GPT2, "gemv_multi"},
    [F_LAYERNORM] = {M_GPT2, "layernorm"},
    [F_GELU] = {M_GPT2, "gelu"},
    [F_ATTN_G1] = {M_GPT2, "attn_decode_g1"},
    [F_GPT2_EMBED] = {M_GPT2, "gpt2_embed"},
    [F_GPT2_LN_QKV] = {M_GPT2, "gpt2_ln_qkv"},
    [F_GPT2_ATTN] = {M_GPT2, "gpt2_attn"},
    [F_GPT2_RESID] = {M_GPT2, "gpt2_gemv_resid"},
    [F_GPT2_LN_FC] = {M_GPT2, "gpt2_ln_fc_gelu"},
    [F_GPT2_LMHEAD] = {M_GPT2, "gpt2_lmhead"},
    [F_GPT2_FINALIZE] = {M_GPT2, "sb_finalize"},
    [F_GEMV_H_B200] = {M_QWEN, "gemv_h_b200"},
    [F_GEMV_HH1] = {M_QWEN, "gemv_hh1"},
    [F_GEMV_HH2] = {M_QWEN, "gemv_hh2"},
    [F_GEMV_HH4] = {M_QWEN, "gemv_hh4"},
    [F_GEMV_HH_SK1] = {M_QWEN, "gemv_hh_sk1"},
    [F_GEMV_HH_SK2] = {M_QWEN, "gemv_hh_sk2"},
    [F_GEMV_HH_SK4] = {M_QWEN, "gemv_hh_sk4"},
    [F_GEMV_H_SK] = {M_QWEN, "gemv_h_sk"},
    [F_GEMV_F32_SK] = {M_GPT2, "gemv_f32_sk"},
    [F_RMSNORM] = {M_QWEN, "rmsnorm"},
    [F_ROPE] = {M_QWEN, "rope"},
    [F_SWIGLU] = {M_QWEN, "swiglu"},
    [F_ATTN_G7] = {M_QWEN, "attn_decode_g7"},
    [F_QWEN_EMBED] = {M_QWEN, "qwen_embed"},
    [F_QWEN_QKV] = {M_QWEN, "qwen_qkv_rope"},
    [F_QWEN_ATTN] = {M_QWEN, "qwen_attn"},
    [F_QWEN_RESID] = {M_QWEN, "qwen_gemv_resid"},
    [F_QWEN_GATEUP] = {M_QWEN, "qwen_gateup_swiglu"},
    [F_QWEN_LMHEAD] = {M_QWEN, "qwen_lmhead"},
    [F_QWEN_FINALIZE] = {M_QWEN, "sb_finalize"},
    [F_QWEN_MK] = {M_QWEN, "qwen_decode_mk"},
    [F_QWEN_MK2] = {M_QWEN, "qwen_decode_mk2"},
    [F_TRANSPOSE_U16] = {M_QWEN, "transpose_u16"},
    [F_FP16_FLUSH] = {M_QWEN, "fp16_flush_subnormals"},
    [F_GEMM_HH_TC] = {M_TC, "gemm_hh_tc"},
    [F_SPLITK_REDUCE] = {M_TC, "gemm_splitk_reduce"},
    [F_SPLITK_REDUCE4] = {M_TC, "gemm_splitk_reduce4"},
    [F_SGEMM_3XTF32] = {M_TC, "sgemm_3xtf32_tc"},
    [F_SGEMM_3XTF32_DST] = {M_TC, "sgemm_3xtf32_tc_dst"},
    [F_TRANSPOSE_F32] = {M_TC, "transpose_f32"},
    [F_PF_EMBED] = {M_QWEN, "qwen_pf_embed"},
    [F_PF_RMS_SPLIT] = {M_QWEN, "qwen_pf_rms_split"},
    [F_PF_SPLIT] = {M_QWEN, "qwen_pf_split"},
    [F_PF_QKV] = {M_QWEN, "qwen_pf_qkv"},
    [F_PF_ATTN] = {M_QWEN, "qwen_pf_attn"},
    [F_PF_RESID] = {M_QWEN, "qwen_pf_resid"},
    [F_PF_SWIGLU_SPLIT] = {M_QWEN, "qwen_pf_swiglu_split"},
    [F_G2PF_EMBED] = {M_GPT2, "gpt2_pf_embed"},
    [F_G2PF_QKV] = {M_GPT2, "gpt2_pf_qkv"},
    [F_G2PF_BIAS_RESID] = {M_GPT2, "gpt2_pf_bias_resid"},
    [F_G2PF_BIAS_GELU] = {M_GPT2, "gpt2_pf_bias_gelu"},
    [F_G2_LAYERNORM_ROWS] = {M_GPT2, "layernorm"},
    [F_GPT2_MK] = {M_GPT2, "gpt2_decode_mk"},
};

/* ---------------------------------------------------------------- errors */
static __thread char err_msg[512];

int sb_fail(int code, const char *what, const char *file, int line) {
    const char *s = NULL;
    if (code < SB_ERR_ARG) cuGetErrorString((CUresult)code, &s);
    const char *base = strrchr(file, '/');
    snprintf(err_msg, sizeof err_msg, "%s (%d%s%s) at %s:%d", what, code, s ? ": " : "", s ? s : "",
             base ? base + 1 : file, line);
    return code;
}

const char *sb_last_error(void) { return err_msg; }

/* ---------------------------------------------------------------- contexts */
#define SB_MAX_CTX 16
static sb_ctx ctxs[SB_MAX_CTX];
static int nctx;
static pthread_mutex_t ctx_lock = PTHREAD_MUTEX_INITIALIZER;

static int ensure_current(int device) {
    SB_CK(cuInit(0));
    CUcontext cur = NULL;
    SB_CK(cuCtxGetCurrent(&cur));
    if (cur) return 0;
    CUdevice dev;
    SB_CK(cuDeviceGet(&dev, device));
    SB_CK(cuDevicePrimaryCtxRetain(&cur, dev));
    SB_CK(cuCtxSetCurrent(cur));
    return 0;
}

static int load_modules(sb_ctx *c) {
    for (int m = 0; m < M_COUNT; m++) SB_CK(cuModuleLoadData(&c->mod[m], images[m].lo));
    SB_CK(cuCtxGetDevice(&c->dev));
    SB_CK(cuDeviceGetAttribute(&c->sms, CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, c->dev));
    return 0;
}

sb_ctx *sb_ctx_get(void) {
    if (ensure_current(0)) return NULL;
    CUcontext cur = NULL;
    if (cuCtxGetCurrent(&cur) != CUDA_SUCCESS || !cur) {
        sb_fail(SB_ERR_STATE, "no current CUDA context", __FILE__, __LINE__);
        return NULL;
    }
    /* keyed by the context's id, not its handle: a context created after
     * another was destroyed may reuse the old handle value */
    unsigned long long id = 0;
    if (cuCtxGetId(cur, &id) != CUDA_SUCCESS) {
        sb_fail(SB_ERR_STATE, "cuCtxGetId", __FILE__, __LINE__);
        return NULL;
    }
    pthread_mutex_lock(&ctx_lock);
    sb_ctx *found = NULL;
    for (int i = 0; i < nctx; i++)
        if (ctxs[i].ctx_id == id) found = &ctxs[i];
    if (!found && nctx < SB_MAX_CTX) {
        sb_ctx *c = &ctxs[nctx];
        memset(c, 0, sizeof *c);
        c->ctx = cur;
        c->ctx_id = id;
        if (load_modules(c) == 0) { found = c; nctx++; }
    } else if (!found) {
        sb_fail(SB_ERR_STATE, "too many CUDA contexts", __FILE__, __LINE__);
    }
    pthread_mutex_unlock(&ctx_lock);
    return found;
}

int sb_init(int device) {
    int rc = ensure_current(device);
    if (rc) return rc;
    return sb_ctx_get() ? 0 : SB_ERR_STATE;
}

int sb_sm_count(void) {
    sb_ctx *c = sb_ctx_get();
    return c ? c->sms : 0;
}

int sb_module_image(const char *name, const void **image, size_t *size) {
    for (int m = 0; m < M_COUNT; m++)
        if (!strcmp(name, images[m].name)) {
            *image = images[m].lo;
            *size = (size_t)(images[m].hi - images[m].lo);
            return 0;
        }
    return sb_fail(SB_ERR_ARG, "unknown module image", __FILE__, __LINE__);
}

/* ---------------------------------------------------------------- launches */
int sb_launch(sb_ctx *c, sb_fn_id f, unsigned gx, unsigned gy, unsigned bx, unsigned smem, CUstream s,
              void **args, int pdl) {
    if (!c->fn[f]) SB_CK(cuModuleGetFunction(&c->fn[f], c->mod[fn_table[f].mod], fn_table[f].name));
    if (smem > 48 * 1024 && c->smem_set[f] < (int)smem) {
        SB_CK(cuFuncSetAttribute(c->fn[f], CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)smem));
        c->smem_set[f] = (int)smem;
    }
    if (gx == 0 || gy == 0) return 0;
    if (!pdl) {
        SB_CK(cuLaunchKernel(c->fn[f], gx, gy, 1, bx, 1, 1, smem, s, args, NULL));
        return 0;
    }
    CUlaunchAttribute attr;
    memset(&attr, 0, sizeof attr);
    attr.id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attr.value.programmaticStreamSerializationAllowed = 1;
    CUlaunchConfig cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDimX = gx;
    cfg.gridDimY = gy;
    cfg.gridDimZ = 1;
    cfg.blockDimX = bx;
    cfg.blockDimY = 1;
    cfg.blockDimZ = 1;
    cfg.sharedMemBytes = smem;
    cfg.hStream = s;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    SB_CK(cuLaunchKernelEx(&cfg, c->fn[f], args, NULL));
    return 0;
}

/* plain launch on a 3-D grid (no dynamic shared memory, no PDL) */
int sb_launch3(sb_ctx *c, sb_fn_id f, unsigned gx, unsigned gy, unsigned gz, unsigned bx, CUstream s, void **args) {
    if (!c->fn[f]) SB_CK(cuModuleGetFunction(&c->fn[f], c->mod[fn_table[f].mod], fn_table[f].name));
    if (gx == 0 || gy == 0 || gz == 0) return 0;
    SB_CK(cuLaunchKernel(c->fn[f], gx, gy, gz, bx, 1, 1, 0, s, args, NULL));
    return 0;
}

static int resolve(sb_ctx *c, sb_fn_id f, unsigned smem) {
    if (!c->fn[f]) SB_CK(cuModuleGetFunction(&c->fn[f], c->mod[fn_table[f].mod], fn_table[f].name));
    if (smem > 48 * 1024 && c->smem_set[f] < (int)smem) {
        SB_CK(cuFuncSetAttribute(c->fn[f], CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)smem));
        c->smem_set[f] = (int)smem;
    }
    return 0;
}

int sb_occupancy(sb_ctx *c, sb_fn_id f, int block, size_t smem) {
    int n = 0;
    if (resolve(c, f, (unsigned)smem)) return 0;
    if (cuOccupancyMaxActiveBlocksPerMultiprocessor(&n, c->fn[f], block, smem) != CUDA_SUCCESS) return 0;
    return n;
}

int sb_launch_coop(sb_ctx *c, sb_fn_id f, unsigned gx, unsigned bx, unsigned smem, CUstream s, void **args) {
    int rc = resolve(c, f, smem);
    if (rc) return rc;
    CUlaunchAttribute attr;
    memset(&attr, 0, sizeof attr);
    attr.id = CU_LAUNCH_ATTRIBUTE_COOPERATIVE;
    attr.value.cooperative = 1;
    CUlaunchConfig cfg;
    memset(&cfg, 0, sizeof cfg);
    cfg.gridDimX = gx;
    cfg.gridDimY = 1;
    cfg.gridDimZ = 1;
    cfg.blockDimX = bx;
    cfg.blockDimY = 1;
    cfg.blockDimZ = 1;
    cfg.sharedMemBytes = smem;
    cfg.hStream = s;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    SB_CK(cuLaunchKernelEx(&cfg, c->fn[f], args, NULL));
    return 0;
}
