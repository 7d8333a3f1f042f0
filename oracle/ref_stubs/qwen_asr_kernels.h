/* Stub for compiling the reference's src/tts_vocoder_ops.c alone (test
 * infrastructure): that file includes the kernels header but calls nothing
 * from it. */
#ifndef LAI_STUB_QWEN_ASR_KERNELS_H
#define LAI_STUB_QWEN_ASR_KERNELS_H
#endif
