/*
 * Runtime controls of libqwen_b200.so shared by the drop-in libraries and the engine. No counterpart in
 * the reference, whose host libraries have no runtime state: these replace its compile-time constants
 * (hls/common/qwen2_model_config.h:21, kDefaultPrefillSeqTile) and add the error text that a GPU
 * implementation needs.
 */
#ifndef QWEN_B200_RUNTIME_H
#define QWEN_B200_RUNTIME_H

#ifdef __cplusplus
extern "C" {
#endif

/* Text of the last failure on the calling thread (status 30 or 31), "" when none. */
const char* qwen_b200_last_error(void);
/* Prefill sequence capacity (reference: kDefaultPrefillSeqTile = 128, compiled in). Default 128, or
 * QWEN_B200_PREFILL_SEQ_CAPACITY from the environment. */
int qwen_b200_prefill_seq_capacity(void);
/* Set the prefill capacity (1..32768); returns 0, or 1 for an out-of-range value. */
int qwen_b200_set_prefill_seq_capacity(int capacity);
/* Error flag of the streaming kernels on the current device: 0 = none, 1 = a pipeline wait gave up after
 * its bounded timeout (the kernel ended early instead of hanging). reset != 0 clears it. */
unsigned qwen_b200_kernel_error(int reset);
/* Number of visible CUDA devices (0 when the driver or device is absent). */
int qwen_b200_device_count(void);

#ifdef __cplusplus
}
#endif

#endif /* QWEN_B200_RUNTIME_H */
