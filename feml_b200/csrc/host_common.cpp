#include "host_common.h"

#include <cstring>

namespace fb {

static thread_local std::string g_last_error;

int set_error(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

const char *last_error() { return g_last_error.c_str(); }

// Same rows, same order as the reference table (feml-core/src/dtype.rs:52-72):
// the order is the DType discriminant, so it is an interface, not a choice.
static const DTypeTraits kTable[FB_DTYPE_COUNT] = {
    {"i8", 1, 1, false},     {"i16", 1, 2, false},    {"i32", 1, 4, false},
    {"i64", 1, 8, false},    {"f16", 1, 2, false},    {"f32", 1, 4, false},
    {"f64", 1, 8, false},    {"q4_0", 32, 18, true},  {"q4_1", 32, 20, true},
    {"q5_0", 32, 22, true},  {"q5_1", 32, 24, true},  {"q8_0", 32, 34, true},
    {"q8_1", 32, 36, true},  {"q2_k", 256, 84, true}, {"q3_k", 256, 110, true},
    {"q4_k", 256, 144, true}, {"q5_k", 256, 176, true}, {"q6_k", 256, 210, true},
    {"q8_k", 256, 292, true},
};

const DTypeTraits *dtype_traits(int32_t dtype) {
    if (dtype < 0 || dtype >= FB_DTYPE_COUNT) return nullptr;
    return &kTable[dtype];
}

int64_t row_size(int32_t dtype, int64_t n) {
    const DTypeTraits *t = dtype_traits(dtype);
    if (!t || n < 0 || n % t->block_size != 0) return -1;
    return t->type_size * (n / t->block_size);
}

const char *op_name(int32_t op) {
    static const char *names[] = {"none",    "view",     "mul",  "add",      "mul_mat",
                                  "mul_mat_id", "rms_norm", "softmax", "rope", "silu",
                                  "get_rows", "concat",  "copy", "diag_mask_inf", "scale"};
    if (op < 0 || op > FB_OP_SCALE) return "unknown";
    return names[op];
}

}  // namespace fb

extern "C" const char *feml_b200_last_error(void) { return fb::last_error(); }
extern "C" const char *feml_b200_version(void) { return "feml_b200 0.1.0 (sm_100a)"; }
