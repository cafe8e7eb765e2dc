// Compile-only host stand-in for the reference's Tensor<T> container
// (include/core/Tensor.cuh in the reference). It lets the reference's test
// sources be compiled in place so that their CPU helper functions can be
// called; the test bodies that use it are never executed. Test
// infrastructure, not product code.
#pragma once

#include <cstdlib>
#include <vector>
#include <numeric>
#include <functional>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <common/macro.h>

enum DeviceType
{
    CPU_PINNED,
    CPU,
    GPU
};

template <typename T>
class Tensor
{
public:
    explicit Tensor(const std::vector<unsigned int> &shape, DeviceType devtype = CPU)
        : shape_(shape), devtype_(devtype),
          size_(std::accumulate(shape.begin(), shape.end(), 1u, std::multiplies<unsigned int>())),
          data_(static_cast<T *>(std::calloc(size_ ? size_ : 1, sizeof(T))))
    {
    }
    ~Tensor() { std::free(data_); }
    Tensor(const Tensor &) = delete;
    Tensor &operator=(const Tensor &) = delete;

    T *data() { return data_; }
    const T *data() const { return data_; }
    unsigned int numel() const { return size_; }
    unsigned int ndim() const { return static_cast<unsigned int>(shape_.size()); }
    const std::vector<unsigned int> &shape() const { return shape_; }
    DeviceType devtype() const { return devtype_; }
    bool empty() const { return size_ == 0; }

private:
    std::vector<unsigned int> shape_;
    DeviceType devtype_;
    unsigned int size_;
    T *data_;
};
