/* distrain-b200 C ABI: the training engine for callers that are not Python programs.
 *
 * Same function set, argument order and JSON replies as the reference's FFI header
 * (node/ffi/distrain.h), so a C, Swift or Kotlin caller written against it can switch libraries.
 * Every char* result is a JSON text allocated by this library; release it with
 * distrain_free_string. Failures come back as {"error": "..."}.
 *
 * The engine runs on the Python interpreter already in the process (when the library is loaded
 * from Python) or on one the library starts on first use (when a C program links it; set
 * DT_LIBPYTHON to the libpython to load and DT_PYTHONPATH to extra module directories if the
 * defaults recorded at build time do not apply). Calls are serialised by one lock and take the
 * interpreter lock themselves, so Python callers must not hold it across a call: ctypes.CDLL releases
 * it during foreign calls (use that, not ctypes.PyDLL).
 * distrain_compute_shard_assignment and distrain_cosine_lr are native and need no interpreter. */
#ifndef DISTRAIN_C_H
#define DISTRAIN_C_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void distrain_set_backend(uint8_t use_gpu);               /* 1: CUDA device 0 when present, 0: CPU */
char* distrain_init(const char* preset);                  /* "MicroTest" | "Tiny" | "Small" | "Medium" | "Large" */
char* distrain_load_shards(const char* paths_json, size_t batch_size, size_t seq_len);
char* distrain_train_step(double learning_rate);          /* {loss, step, tokens_processed} */
char* distrain_status(void);                              /* {initialized, step, last_loss, total_tokens, model_preset, gpu} */
char* distrain_calibrate(double target_interval_secs);    /* {secs_per_step, recommended_h_mini} */
char* distrain_load_checkpoint_file(const char* path);    /* safetensors file */
char* distrain_load_checkpoint(const uint8_t* data, size_t len);
char* distrain_snapshot_params(void);
char* distrain_compute_delta(const char* output_path);    /* zstd JSON SparseDelta of snapshot - current */
char* distrain_compute_shard_assignment(const char* node_id, uint64_t version, uint32_t total_shards,
                                        uint32_t shards_per_node);
char* distrain_default_training_params(void);
double distrain_cosine_lr(uint64_t step, uint64_t warmup_steps, uint64_t total_steps, double max_lr,
                          double min_lr);
void distrain_shutdown(void);
void distrain_free_string(char* ptr);

#ifdef __cplusplus
}
#endif
#endif
