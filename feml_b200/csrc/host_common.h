// Host-side helpers shared by the C++ graph mirror and the B200 backend:
// thread-local error reporting and the ggml dtype size table.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/feml_b200.h"

namespace fb {

// Record `msg` as the calling thread's last error and return `code`.
int set_error(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
const char *last_error();

// ggml blck_size / type_size table, indexed by DType discriminant
// (feml-core/src/dtype.rs:52-72).
struct DTypeTraits {
    const char *name;
    int64_t block_size;
    int64_t type_size;
    bool quantized;
};
const DTypeTraits *dtype_traits(int32_t dtype);  // nullptr when out of range

// Row bytes of `n` elements (DType::row_size, dtype.rs:105-116); -1 when n is
// not a multiple of the block size or the dtype is unknown.
int64_t row_size(int32_t dtype, int64_t n);

const char *op_name(int32_t op);

}  // namespace fb
