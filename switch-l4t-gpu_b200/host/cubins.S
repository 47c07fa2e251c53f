/* cubins.S -- links the five sm_100a module images into libswitch_b200.so
 * (found on the assembler include path, i.e. the build's lib/ directory). */
        .section .rodata
#define SB_IMAGE(sym, file)     \
        .balign 64;             \
        .global sym;            \
sym:    .incbin file;           \
        .byte 0;                \
        .global sym##_end;      \
sym##_end:

SB_IMAGE(sb_img_switch_gpu, "switch_gpu.cubin")
SB_IMAGE(sb_img_gemv, "gemv.cubin")
SB_IMAGE(sb_img_gpt2, "gpt2.cubin")
SB_IMAGE(sb_img_qwen, "qwen.cubin")
SB_IMAGE(sb_img_tc, "tc.cubin")

        .section .note.GNU-stack,"",@progbits
