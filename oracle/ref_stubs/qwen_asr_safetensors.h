/* Stub for compiling the reference's src/tts_vocoder_ops.c alone (test
 * infrastructure). The real header lives in the un-vendored qwen-asr
 * submodule; tts_vocoder.h only needs this opaque type name. */
#ifndef LAI_STUB_QWEN_ASR_SAFETENSORS_H
#define LAI_STUB_QWEN_ASR_SAFETENSORS_H
typedef struct multi_safetensors multi_safetensors_t;
#endif
