/* sb_internal.h -- private declarations of libswitch_b200 (driver-API host). */
#ifndef SB_INTERNAL_H
#define SB_INTERNAL_H
#include <cuda.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/switch_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

enum { M_SWITCH = 0, M_GEMV, M_GPT2, M_QWEN, M_TC, M_COUNT };

typedef enum {
    F_SGEMM_B200 = 0,
    F_SGEMM_B200_DST,
    F_SGEMM_B200_STK,
    F_SGEMM_STK_FIXUP,
    F_SGEMM_TMA,
    F_GEMM_HH_MMA8,
    F_GEMM_HH_MMA16,
    F_GEMM_HH_MMA8_W4,
    F_GEMM_HH_MMA16_W4,
    F_TOPK_PARTIAL,
    F_SPLITK_REDUCE4,
    F_TOPK_MERGE,
    F_SGEMM_NAIVE,
    F_MEMBW,
    F_FMA_PEAK,
    F_GEMV_F32_B200,
    F_GEMV_MULTI,
    F_LAYERNORM,
    F_GELU,
    F_ATTN_G1,
    F_GPT2_EMBED,
    F_GPT2_LN_QKV,
    F_GPT2_ATTN,
    F_GPT2_RESID,
    F_GPT2_LN_FC,
    F_GPT2_LMHEAD,
    F_GPT2_FINALIZE,
    F_GEMV_H_B200,
    F_GEMV_HH1,
    F_GEMV_HH2,
    F_GEMV_HH4,
    F_GEMV_HH_SK1,
    F_GEMV_HH_SK2,
    F_GEMV_HH_SK4,
    F_GEMV_H_SK,
    F_GEMV_F32_SK,
    F_RMSNORM,
    F_ROPE,
    F_SWIGLU,
    F_ATTN_G7,
    F_QWEN_EMBED,
    F_QWEN_QKV,
    F_QWEN_ATTN,
    F_QWEN_RESID,
    F_QWEN_GATEUP,
    F_QWEN_LMHEAD,
    F_QWEN_FINALIZE,
    F_QWEN_MK,
    F_QWEN_MK2,
    F_TRANSPOSE_U16,
    F_FP16_FLUSH,
    F_GEMM_HH_TC,
    F_SPLITK_REDUCE,
    F_SGEMM_3XTF32,
    F_SGEMM_3XTF32_DST,
    F_TRANSPOSE_F32,
    F_PF_EMBED,
    F_PF_RMS_SPLIT,
    F_PF_SPLIT,
    F_PF_QKV,
    F_PF_ATTN,
    F_PF_RESID,
    F_PF_SWIGLU_SPLIT,
    F_G2PF_EMBED,
    F_G2PF_QKV,
    F_G2PF_BIAS_RESID,
    F_G2PF_BIAS_GELU,
    F_G2_LAYERNORM_ROWS,
    F_GPT2_MK,
    F_COUNT
} sb_fn_id;

typedef struct sb_ctx {
    CUcontext ctx;
    unsigned long long ctx_id; /* cuCtxGetId: unique for the process's life */
    CUdevice dev;
    CUmodule mod[M_COUNT];
    CUfunction fn[F_COUNT];
    int smem_set[F_COUNT]; /* dynamic smem limit already raised to this */
    int sms;
    CUdeviceptr tc_ws; /* split-K workspace of the tensor-core GEMM (grown on demand) */
    size_t tc_ws_bytes;
    CUdeviceptr tc_bt; /* K-major copy of B for the 3xTF32 SGEMM (grown on demand) */
    size_t tc_bt_bytes;
} sb_ctx;

/* error reporting (thread-local message) */
int sb_fail(int code, const char *what, const char *file, int line);
#define SB_CK(call)                                                           \
    do {                                                                      \
        CUresult r_ = (call);                                                 \
        if (r_ != CUDA_SUCCESS) return sb_fail((int)r_, #call, __FILE__, __LINE__); \
    } while (0)
#define SB_ARG(cond, msg)                                                     \
    do {                                                                      \
        if (!(cond)) return sb_fail(SB_ERR_ARG, msg, __FILE__, __LINE__);     \
    } while (0)

/* current-context state (modules loaded); NULL on failure (error recorded) */
sb_ctx *sb_ctx_get(void);
/* launch fn with grid/block/dynamic smem on stream; pdl != 0 adds the
 * programmatic stream-serialisation attribute */
int sb_launch(sb_ctx *c, sb_fn_id f, unsigned gx, unsigned gy, unsigned bx, unsigned smem, CUstream s,
              void **args, int pdl);
/* cooperative launch (all CTAs co-resident, required by grid-wide barriers) */
int sb_launch_coop(sb_ctx *c, sb_fn_id f, unsigned gx, unsigned bx, unsigned smem, CUstream s, void **args);
int sb_launch3(sb_ctx *c, sb_fn_id f, unsigned gx, unsigned gy, unsigned gz, unsigned bx, CUstream s, void **args);
/* max co-resident CTAs of f per SM at this block size / dynamic smem */
int sb_occupancy(sb_ctx *c, sb_fn_id f, int block, size_t smem);

#ifdef __cplusplus
}
#endif
#endif
