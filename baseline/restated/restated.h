/* The reference's per-step GPU forward restated in CUDA C++ (restated.cu): the latency baseline
 * this library is compared with on the same GPU. Not part of the product's boundary. */
#ifndef JC_RESTATED_H
#define JC_RESTATED_H
#include <stddef.h>
#include <stdint.h>

#include "../../include/julia_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Prepares raw weights (the format of julia_cuda_raw_size) in the reference's layouts (folded
 * LayerNorms, RoPE-permuted Wqkv, fragment-interleaved Wi) on GPU `device`, buffers for up to
 * max_length tokens (0: max_positions). NULL with a message in err on failure. */
void *jc_restated_load(const jc_model_config *cfg, const float *raw, size_t raw_len, size_t max_length,
                       int device, char *err, size_t err_len);

/* One request: n token ids, n_markers marker rows, question type qtype; logits one per marker,
 * gpu_ms the CUDA-event time embed -> logits. 0, or -1 with a message in err. */
int jc_restated_run(void *handle, const uint32_t *ids, size_t n, const uint32_t *markers, size_t n_markers,
                    uint32_t qtype, float *logits, float *gpu_ms, char *err, size_t err_len);

void jc_restated_free(void *handle);

#ifdef __cplusplus
}
#endif
#endif
