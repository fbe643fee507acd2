// ggml_host.cpp -- TEST INFRASTRUCTURE ONLY: host-only implementation of the
// ggml names declared in this directory, linked with the reference's own
// decoder sources into oracle/_ref/libref_decoder.so (the parity checker).
//
// What runs on the decoder's CPU branch is implemented: tensor element and
// byte counts, ggml_backend_tensor_get/set as host copies, a CPU backend
// device, and to_float for F32 / F16 / Q8_0 written from the public GGUF block
// formats (F16: IEEE-754 binary16; Q8_0: 32-weight blocks {binary16 d;
// int8 qs[32]}, value d * qs[i]). The binary16 decode here is computed with
// ldexp, independently of the bit-assembly decode in oracle.cpp, so that the
// two checkers do not share a mistake. Every graph, allocator and compute call
// aborts: the CPU branch (`use_graphs == false`) never makes one, and reaching
// one would mean the reference took its GPU branch.

#include "ggml.h"
#include "ggml-alloc.h"
#include "ggml-backend.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace {

[[noreturn]] void unreachable(const char * what) {
    std::fprintf(stderr, "ggml_host: %s called; only the decoder's CPU branch is supported\n", what);
    std::abort();
}

float binary16_value(uint16_t h) {
    const int sign = (h >> 15) & 1;
    const int e = (h >> 10) & 0x1F;
    const int m = h & 0x3FF;
    float v;
    if (e == 0x1F) {
        v = m ? NAN : INFINITY;
    } else if (e == 0) {
        v = std::ldexp((float) m, -24);                  // subnormal: m * 2^-24
    } else {
        v = std::ldexp((float) (1024 + m), e - 25);      // (1 + m/1024) * 2^(e-15)
    }
    return sign ? -v : v;
}

void f16_to_float(const void * x, float * y, int64_t k) {
    const uint8_t * p = static_cast<const uint8_t *>(x);
    for (int64_t i = 0; i < k; ++i) {
        uint16_t h;
        std::memcpy(&h, p + 2 * i, 2);
        y[i] = binary16_value(h);
    }
}

void q8_0_to_float(const void * x, float * y, int64_t k) {
    const uint8_t * p = static_cast<const uint8_t *>(x);
    for (int64_t b = 0; b < k / 32; ++b) {
        uint16_t dh;
        std::memcpy(&dh, p + 34 * b, 2);
        const float d = binary16_value(dh);
        const int8_t * qs = reinterpret_cast<const int8_t *>(p + 34 * b + 2);
        for (int j = 0; j < 32; ++j) y[32 * b + j] = d * (float) qs[j];
    }
}

void f32_to_float(const void * x, float * y, int64_t k) { std::memcpy(y, x, (size_t) k * 4); }

const ggml_type_traits k_f32  = {"f32", 1, 4, false, f32_to_float};
const ggml_type_traits k_f16  = {"f16", 1, 2, false, f16_to_float};
const ggml_type_traits k_q8_0 = {"q8_0", 32, 34, true, q8_0_to_float};
const ggml_type_traits k_i32  = {"i32", 1, 4, false, nullptr};

// The single backend: a CPU device.
struct host_object { int tag; };
host_object g_backend{1}, g_device{2}, g_reg{3};

}  // namespace

extern "C" {

const ggml_type_traits * ggml_get_type_traits(enum ggml_type type) {
    switch (type) {
        case GGML_TYPE_F32:  return &k_f32;
        case GGML_TYPE_F16:  return &k_f16;
        case GGML_TYPE_Q8_0: return &k_q8_0;
        case GGML_TYPE_I32:  return &k_i32;
        default:             return nullptr;
    }
}

const char * ggml_type_name(enum ggml_type type) {
    const ggml_type_traits * t = ggml_get_type_traits(type);
    return t ? t->type_name : "unsupported";
}

int64_t ggml_nelements(const ggml_tensor * t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

size_t ggml_nbytes(const ggml_tensor * t) {
    const ggml_type_traits * tr = ggml_get_type_traits(t->type);
    if (!tr) return 0;
    // rows of ne[0] elements stored as ne[0] / blck_size blocks, strided by nb[1..3]
    size_t n = (size_t) (t->ne[0] / tr->blck_size) * tr->type_size;
    for (int i = 1; i < GGML_MAX_DIMS; ++i) n += (size_t) (t->ne[i] - 1) * t->nb[i];
    return n;
}

size_t ggml_tensor_overhead(void) { return sizeof(ggml_tensor); }
size_t ggml_graph_overhead_custom(size_t, bool) { return 0; }
void   ggml_log_set(ggml_log_callback, void *) {}

ggml_context * ggml_init(ggml_init_params) { unreachable("ggml_init"); }
void ggml_free(ggml_context * ctx) { if (ctx) unreachable("ggml_free"); }

ggml_tensor * ggml_new_tensor_1d(ggml_context *, enum ggml_type, int64_t) { unreachable("ggml_new_tensor_1d"); }
ggml_tensor * ggml_new_tensor_2d(ggml_context *, enum ggml_type, int64_t, int64_t) { unreachable("ggml_new_tensor_2d"); }
ggml_tensor * ggml_set_name(ggml_tensor *, const char *) { unreachable("ggml_set_name"); }
void ggml_set_input(ggml_tensor *) { unreachable("ggml_set_input"); }
void ggml_set_output(ggml_tensor *) { unreachable("ggml_set_output"); }
ggml_tensor * ggml_get_rows(ggml_context *, ggml_tensor *, ggml_tensor *) { unreachable("ggml_get_rows"); }
ggml_tensor * ggml_reshape_1d(ggml_context *, ggml_tensor *, int64_t) { unreachable("ggml_reshape_1d"); }
ggml_tensor * ggml_view_1d(ggml_context *, ggml_tensor *, int64_t, size_t) { unreachable("ggml_view_1d"); }
ggml_tensor * ggml_view_2d(ggml_context *, ggml_tensor *, int64_t, int64_t, size_t, size_t) { unreachable("ggml_view_2d"); }
ggml_tensor * ggml_mul_mat(ggml_context *, ggml_tensor *, ggml_tensor *) { unreachable("ggml_mul_mat"); }
ggml_tensor * ggml_add(ggml_context *, ggml_tensor *, ggml_tensor *) { unreachable("ggml_add"); }
ggml_tensor * ggml_mul(ggml_context *, ggml_tensor *, ggml_tensor *) { unreachable("ggml_mul"); }
ggml_tensor * ggml_sigmoid(ggml_context *, ggml_tensor *) { unreachable("ggml_sigmoid"); }
ggml_tensor * ggml_tanh(ggml_context *, ggml_tensor *) { unreachable("ggml_tanh"); }
ggml_tensor * ggml_relu(ggml_context *, ggml_tensor *) { unreachable("ggml_relu"); }
ggml_tensor * ggml_cont(ggml_context *, ggml_tensor *) { unreachable("ggml_cont"); }
ggml_tensor * ggml_cpy(ggml_context *, ggml_tensor *, ggml_tensor *) { unreachable("ggml_cpy"); }
ggml_tensor * ggml_argmax(ggml_context *, ggml_tensor *) { unreachable("ggml_argmax"); }
ggml_cgraph * ggml_new_graph_custom(ggml_context *, size_t, bool) { unreachable("ggml_new_graph_custom"); }
void ggml_build_forward_expand(ggml_cgraph *, ggml_tensor *) { unreachable("ggml_build_forward_expand"); }

ggml_backend_dev_t ggml_backend_get_device(ggml_backend_t b) {
    return b ? reinterpret_cast<ggml_backend_dev_t>(&g_device) : nullptr;
}
enum ggml_backend_dev_type ggml_backend_dev_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_CPU; }
ggml_backend_reg_t ggml_backend_dev_backend_reg(ggml_backend_dev_t) { return reinterpret_cast<ggml_backend_reg_t>(&g_reg); }
const char * ggml_backend_reg_name(ggml_backend_reg_t) { return "CPU"; }
void * ggml_backend_reg_get_proc_address(ggml_backend_reg_t, const char *) { return nullptr; }

void ggml_backend_tensor_get(const ggml_tensor * t, void * data, size_t offset, size_t size) {
    if (offset + size > ggml_nbytes(t)) unreachable("ggml_backend_tensor_get out of range");
    std::memcpy(data, static_cast<const uint8_t *>(t->data) + offset, size);
}
void ggml_backend_tensor_set(ggml_tensor * t, const void * data, size_t offset, size_t size) {
    if (offset + size > ggml_nbytes(t)) unreachable("ggml_backend_tensor_set out of range");
    std::memcpy(static_cast<uint8_t *>(t->data) + offset, data, size);
}
void ggml_backend_tensor_memset(ggml_tensor *, uint8_t, size_t, size_t) { unreachable("ggml_backend_tensor_memset"); }

ggml_backend_buffer_type_t ggml_backend_get_default_buffer_type(ggml_backend_t) { unreachable("ggml_backend_get_default_buffer_type"); }
void ggml_backend_buffer_free(ggml_backend_buffer_t b) { if (b) unreachable("ggml_backend_buffer_free"); }
enum ggml_status ggml_backend_graph_compute(ggml_backend_t, ggml_cgraph *) { unreachable("ggml_backend_graph_compute"); }

ggml_gallocr_t ggml_gallocr_new(ggml_backend_buffer_type_t) { unreachable("ggml_gallocr_new"); }
void ggml_gallocr_free(ggml_gallocr_t g) { if (g) unreachable("ggml_gallocr_free"); }
bool ggml_gallocr_alloc_graph(ggml_gallocr_t, ggml_cgraph *) { unreachable("ggml_gallocr_alloc_graph"); }
ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(ggml_context *, ggml_backend_t) { unreachable("ggml_backend_alloc_ctx_tensors"); }

}  // extern "C"

// The backend handle the shim hands to the model (ParakeetCtcModel::backend_active).
ggml_backend_t ggml_host_cpu_backend() { return reinterpret_cast<ggml_backend_t>(&g_backend); }
