// Scalar typedefs and element types of QuasarML (QuasarML/src/Common/Types.h),
// kept identical so user code compiles unchanged.  The DataType order and
// sizes are also the QSML_* codes of include/qsml_cuda.h.
#pragma once

#include <cstddef>
#include <cstdint>

namespace QuasarML {

using u8 = uint8_t;
using u16 = uint16_t;
using u32 = uint32_t;
using u64 = uint64_t;
using i8 = int8_t;
using i16 = int16_t;
using i32 = int32_t;
using i64 = int64_t;
using f32 = float;
using f64 = double;
using b8 = bool;
using b32 = int32_t;

#define QS_API __attribute__((visibility("default")))

enum class DataType : u32 { F32 = 0, F16, I32, I16, I8, U32, U16, U8 };

constexpr u32 dtype_size(DataType dtype) {
    switch (dtype) {
        case DataType::F32: case DataType::I32: case DataType::U32: return 4;
        case DataType::F16: case DataType::I16: case DataType::U16: return 2;
        case DataType::I8: case DataType::U8: return 1;
    }
    return 0;
}

QS_API const char* dtype_to_string(DataType dtype);

}  // namespace QuasarML
