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

/* One restated GEMM on device pointers (the reference's gemm_* kernel arguments, kernels/src/
 * main.rs:1043-1066, tile and split by gemm::choose with `sms` SMs; epi one of the eight JC_EPI_*
 * combinations of the forward; the rope table natural [rows][32][2]), queued on `stream`. With
 * split-K, ws and counters sized by the two functions below (counters zeroed). 0 or -1. */
size_t jc_restated_gemm_ws_floats(uint32_t m, uint32_t n, uint32_t k, int sms);
size_t jc_restated_gemm_counters(uint32_t m, uint32_t n, uint32_t k, int sms);
int jc_restated_gemm(uint32_t epi, const void *a, const void *w, void *c, const void *res, float *ws,
                     uint32_t *counters, const float *stats_in, const float *colsum, float *stats_out,
                     float *zero, uint32_t zero_len, uint32_t m, uint32_t n, uint32_t k, float eps,
                     const float *rope, const float *bias, int sms, void *stream);
/* The restated attention (qkv [n, 3d] f16, o [n, d] f16, window 0 = global) on `stream`. */
int jc_restated_attention(const void *qkv, void *o, uint32_t n, uint32_t window, uint32_t d, void *stream);

#ifdef __cplusplus
}
#endif
#endif
