/*
 * ggml-backend.h -- TEST INFRASTRUCTURE ONLY: host-only stand-in for the
 * ggml backend API names the reference's decoder sources use (see ggml.h in
 * this directory for why it exists). The one backend it knows is a CPU
 * device whose tensors live in host memory.
 */
#pragma once

#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ggml_backend *             ggml_backend_t;
typedef struct ggml_backend_buffer *      ggml_backend_buffer_t;
typedef struct ggml_backend_buffer_type * ggml_backend_buffer_type_t;
typedef struct ggml_backend_device *      ggml_backend_dev_t;
typedef struct ggml_backend_reg *         ggml_backend_reg_t;

enum ggml_backend_dev_type {
    GGML_BACKEND_DEVICE_TYPE_CPU   = 0,
    GGML_BACKEND_DEVICE_TYPE_GPU   = 1,
    GGML_BACKEND_DEVICE_TYPE_ACCEL = 2
};

typedef void (*ggml_backend_set_n_threads_t)(ggml_backend_t backend, int n_threads);

ggml_backend_dev_t         ggml_backend_get_device(ggml_backend_t backend);
enum ggml_backend_dev_type ggml_backend_dev_type(ggml_backend_dev_t device);
ggml_backend_reg_t         ggml_backend_dev_backend_reg(ggml_backend_dev_t device);
const char *               ggml_backend_reg_name(ggml_backend_reg_t reg);
void *                     ggml_backend_reg_get_proc_address(ggml_backend_reg_t reg, const char * name);

void ggml_backend_tensor_get(const struct ggml_tensor * tensor, void * data, size_t offset, size_t size);
void ggml_backend_tensor_set(struct ggml_tensor * tensor, const void * data, size_t offset, size_t size);
void ggml_backend_tensor_memset(struct ggml_tensor * tensor, uint8_t value, size_t offset, size_t size);

ggml_backend_buffer_type_t ggml_backend_get_default_buffer_type(ggml_backend_t backend);
void                       ggml_backend_buffer_free(ggml_backend_buffer_t buffer);
enum ggml_status           ggml_backend_graph_compute(ggml_backend_t backend, struct ggml_cgraph * cgraph);

#ifdef __cplusplus
}
#endif
