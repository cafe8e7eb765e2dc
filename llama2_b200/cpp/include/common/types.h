// Element and device enums of the C++ operator API (the reference's
// include/common/types.h:53-126, with BF16 added).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

enum DeviceType
{
    CPU_PINNED,
    CPU,
    GPU
};

enum DataType
{
    UNSUPPORTED,
    FP32,
    FP16,
    INT8,
    INT32,
    UINT32,
    BOOL,
    BYTES,
    PTR,
    BF16
};

template <typename T>
struct RealTypeToDataType
{
    static constexpr DataType dtype = UNSUPPORTED;
};
template <> struct RealTypeToDataType<float> { static constexpr DataType dtype = FP32; };
template <> struct RealTypeToDataType<half> { static constexpr DataType dtype = FP16; };
template <> struct RealTypeToDataType<__nv_bfloat16> { static constexpr DataType dtype = BF16; };
template <> struct RealTypeToDataType<int8_t> { static constexpr DataType dtype = INT8; };
template <> struct RealTypeToDataType<int32_t> { static constexpr DataType dtype = INT32; };
template <> struct RealTypeToDataType<uint32_t> { static constexpr DataType dtype = UINT32; };
template <> struct RealTypeToDataType<bool> { static constexpr DataType dtype = BOOL; };
template <> struct RealTypeToDataType<unsigned char> { static constexpr DataType dtype = BYTES; };
template <> struct RealTypeToDataType<void *> { static constexpr DataType dtype = PTR; };
