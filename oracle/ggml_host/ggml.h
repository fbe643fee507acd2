/*
 * ggml.h -- TEST INFRASTRUCTURE ONLY: a host-only stand-in for the parts of
 * ggml's public API that parakeet.cpp's decoder sources name, so that the
 * reference's own src/parakeet_tdt.cpp and src/parakeet_eou.cpp compile
 * unchanged into the parity checker oracle/_ref/libref_decoder.so.
 *
 * ggml itself (ggml-org/ggml, pinned at 58c38058 by the reference's
 * scripts/setup-ggml.sh:32) is an un-vendored dependency absent from this
 * machine. This header declares only names, types and signatures of ggml's
 * public interface; ggml_host.cpp implements what the decoder's CPU branch
 * (`use_graphs == false`, src/parakeet_tdt.cpp:620) runs -- tensor metadata,
 * ggml_backend_tensor_get as a host copy, and to_float for F32 / F16 / Q8_0
 * restated from the public block formats -- and turns every graph-building or
 * backend-compute call into an immediate abort, because the CPU branch never
 * reaches one. The backend it reports is a CPU device, which is what makes
 * tdt_prepare_runtime choose that branch.
 */
#pragma once

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_MAX_DIMS 4
#define GGML_MAX_NAME 64

/* Values are the GGUF wire ids of these types. */
enum ggml_type {
    GGML_TYPE_F32  = 0,
    GGML_TYPE_F16  = 1,
    GGML_TYPE_Q8_0 = 8,
    GGML_TYPE_I32  = 26,
    GGML_TYPE_COUNT = 40
};

enum ggml_status {
    GGML_STATUS_ALLOC_FAILED = -2,
    GGML_STATUS_FAILED       = -1,
    GGML_STATUS_SUCCESS      = 0,
    GGML_STATUS_ABORTED      = 1
};

enum ggml_log_level {
    GGML_LOG_LEVEL_NONE  = 0,
    GGML_LOG_LEVEL_DEBUG = 1,
    GGML_LOG_LEVEL_INFO  = 2,
    GGML_LOG_LEVEL_WARN  = 3,
    GGML_LOG_LEVEL_ERROR = 4,
    GGML_LOG_LEVEL_CONT  = 5
};

typedef void (*ggml_log_callback)(enum ggml_log_level level, const char * text, void * user_data);

struct ggml_context;
struct ggml_cgraph;

/* Only the fields the decoder sources read. */
struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[GGML_MAX_DIMS];   /* elements per dimension, ne[0] contiguous */
    size_t  nb[GGML_MAX_DIMS];   /* strides in bytes */
    void *  data;                /* host bytes of the tensor */
    char    name[GGML_MAX_NAME];
};

struct ggml_init_params {
    size_t mem_size;
    void * mem_buffer;
    bool   no_alloc;
};

typedef void (*ggml_to_float_t)(const void * x, float * y, int64_t k);

struct ggml_type_traits {
    const char *    type_name;
    int64_t         blck_size;
    size_t          type_size;
    bool            is_quantized;
    ggml_to_float_t to_float;
};

const struct ggml_type_traits * ggml_get_type_traits(enum ggml_type type);
const char * ggml_type_name(enum ggml_type type);
int64_t      ggml_nelements(const struct ggml_tensor * tensor);
size_t       ggml_nbytes(const struct ggml_tensor * tensor);
size_t       ggml_tensor_overhead(void);
size_t       ggml_graph_overhead_custom(size_t size, bool grads);
void         ggml_log_set(ggml_log_callback log_callback, void * user_data);

struct ggml_context * ggml_init(struct ggml_init_params params);
void                  ggml_free(struct ggml_context * ctx);

struct ggml_tensor * ggml_new_tensor_1d(struct ggml_context * ctx, enum ggml_type type, int64_t ne0);
struct ggml_tensor * ggml_new_tensor_2d(struct ggml_context * ctx, enum ggml_type type, int64_t ne0, int64_t ne1);
struct ggml_tensor * ggml_set_name(struct ggml_tensor * tensor, const char * name);
void                 ggml_set_input(struct ggml_tensor * tensor);
void                 ggml_set_output(struct ggml_tensor * tensor);

struct ggml_tensor * ggml_get_rows(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b);
struct ggml_tensor * ggml_reshape_1d(struct ggml_context * ctx, struct ggml_tensor * a, int64_t ne0);
struct ggml_tensor * ggml_view_1d(struct ggml_context * ctx, struct ggml_tensor * a, int64_t ne0, size_t offset);
struct ggml_tensor * ggml_view_2d(struct ggml_context * ctx, struct ggml_tensor * a, int64_t ne0, int64_t ne1,
                                  size_t nb1, size_t offset);
struct ggml_tensor * ggml_mul_mat(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b);
struct ggml_tensor * ggml_add(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b);
struct ggml_tensor * ggml_mul(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b);
struct ggml_tensor * ggml_sigmoid(struct ggml_context * ctx, struct ggml_tensor * a);
struct ggml_tensor * ggml_tanh(struct ggml_context * ctx, struct ggml_tensor * a);
struct ggml_tensor * ggml_relu(struct ggml_context * ctx, struct ggml_tensor * a);
struct ggml_tensor * ggml_cont(struct ggml_context * ctx, struct ggml_tensor * a);
struct ggml_tensor * ggml_cpy(struct ggml_context * ctx, struct ggml_tensor * a, struct ggml_tensor * b);
struct ggml_tensor * ggml_argmax(struct ggml_context * ctx, struct ggml_tensor * a);

struct ggml_cgraph * ggml_new_graph_custom(struct ggml_context * ctx, size_t size, bool grads);
void                 ggml_build_forward_expand(struct ggml_cgraph * cgraph, struct ggml_tensor * tensor);

#ifdef __cplusplus
}
#endif
