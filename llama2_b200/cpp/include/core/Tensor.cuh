// Tensor<T>: the owning, typed buffer the operator API passes around, with
// the interface of the reference's include/core/Tensor.cuh:30-334 (shape,
// numel, data, migration between CPU / pinned CPU / GPU, zero-initialized on
// construction). Element counts are 64-bit here (the reference's are 32-bit
// unsigned int, which overflows for caches above 4 G elements). Plain C++ over
// the CUDA runtime API: no kernels in this header.
#pragma once

#include <algorithm>
#include <cassert>
#include <cstdint>
#include <cstring>
#include <functional>
#include <memory>
#include <numeric>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include <cuda_runtime.h>

#include "common/macro.h"
#include "common/types.h"

template <typename T>
class Tensor;

class BaseTensor
{
public:
    BaseTensor(const std::vector<unsigned int> &shape, DataType dtype, DeviceType devtype)
        : shape_(shape), dtype_(dtype), devtype_(devtype)
    {
        size_ = 1;
        for (unsigned int s : shape_)
            size_ *= s;
    }
    virtual ~BaseTensor() = default;
    BaseTensor(const BaseTensor &) = delete;
    BaseTensor &operator=(const BaseTensor &) = delete;
    BaseTensor(BaseTensor &&o) noexcept
        : size_(o.size_), shape_(std::move(o.shape_)), dtype_(o.dtype_), devtype_(o.devtype_)
    {
        o.size_ = 0;
    }
    BaseTensor &operator=(BaseTensor &&o) noexcept
    {
        if (this != &o)
        {
            size_ = o.size_;
            shape_ = std::move(o.shape_);
            dtype_ = o.dtype_;
            devtype_ = o.devtype_;
            o.size_ = 0;
        }
        return *this;
    }

    bool empty() const noexcept { return size_ == 0; }
    uint64_t numel() const noexcept { return size_; }
    unsigned int ndim() const noexcept { return (unsigned int)shape_.size(); }
    const std::vector<unsigned int> &shape() const noexcept { return shape_; }
    DataType dtype() const noexcept { return dtype_; }
    DeviceType devtype() const noexcept { return devtype_; }

    std::vector<uint64_t> strides() const
    {
        std::vector<uint64_t> s(ndim());
        uint64_t st = 1;
        for (int i = (int)ndim() - 1; i >= 0; --i)
        {
            s[i] = st;
            st *= shape_[i];
        }
        return s;
    }

    template <typename U>
    Tensor<U> *as()
    {
        assert(RealTypeToDataType<U>::dtype == dtype_ && "Type mismatch in as<T>()");
        return static_cast<Tensor<U> *>(this);
    }
    template <typename U>
    const Tensor<U> *as() const
    {
        assert(RealTypeToDataType<U>::dtype == dtype_ && "Type mismatch in as<T>()");
        return static_cast<const Tensor<U> *>(this);
    }

protected:
    uint64_t size_;
    std::vector<unsigned int> shape_;
    DataType dtype_;
    DeviceType devtype_;
};

template <typename T>
class Tensor : public BaseTensor
{
public:
    explicit Tensor(const std::vector<unsigned int> &shape, DeviceType devtype = CPU, cudaStream_t stream = 0)
        : BaseTensor(shape, RealTypeToDataType<T>::dtype, devtype), data_(nullptr)
    {
        if (size_ == 0)
            return;
        data_ = allocate(devtype_, size_);
        zero(stream);
    }
    ~Tensor() override { release(); }
    Tensor(const Tensor &) = delete;
    Tensor &operator=(const Tensor &) = delete;
    Tensor(Tensor &&o) noexcept : BaseTensor(std::move(o)), data_(o.data_) { o.data_ = nullptr; }
    Tensor &operator=(Tensor &&o) noexcept
    {
        if (this != &o)
        {
            release();
            BaseTensor::operator=(std::move(o));
            data_ = o.data_;
            o.data_ = nullptr;
        }
        return *this;
    }

    T *data() noexcept { return data_; }
    const T *data() const noexcept { return data_; }

    void to_device(cudaStream_t stream = 0) { migrate(GPU, stream); }
    void to_host() { migrate(CPU, 0); }
    void to_host_pinned(cudaStream_t stream = 0) { migrate(CPU_PINNED, stream); }

    void resize_discard(const std::vector<unsigned int> &shape, cudaStream_t stream = 0)
    {
        Tensor<T> t(shape, devtype_, stream);
        swap(t);
    }

    void swap(Tensor &o) noexcept
    {
        std::swap(size_, o.size_);
        std::swap(shape_, o.shape_);
        std::swap(dtype_, o.dtype_);
        std::swap(devtype_, o.devtype_);
        std::swap(data_, o.data_);
    }

    void constant_val_set(const T &val, cudaStream_t stream = 0)
    {
        if (empty() || !data_)
            return;
        if (devtype_ != GPU)
        {
            std::fill(data_, data_ + size_, val);
            return;
        }
        bool all_zero = true;
        const unsigned char *b = reinterpret_cast<const unsigned char *>(&val);
        for (size_t i = 0; i < sizeof(T); ++i)
            all_zero = all_zero && b[i] == 0;
        if (all_zero)
        {
            CUDA_CHECK(cudaMemsetAsync(data_, 0, size_ * sizeof(T), stream));
            return;
        }
        std::vector<T> host(size_, val);
        CUDA_CHECK(cudaMemcpyAsync(data_, host.data(), size_ * sizeof(T), cudaMemcpyHostToDevice, stream));
        CUDA_CHECK(cudaStreamSynchronize(stream));
    }

private:
    static T *allocate(DeviceType dev, uint64_t n)
    {
        T *p = nullptr;
        switch (dev)
        {
        case CPU_PINNED:
            CUDA_CHECK(cudaHostAlloc((void **)&p, n * sizeof(T), cudaHostAllocDefault));
            break;
        case CPU:
            p = static_cast<T *>(std::malloc(n * sizeof(T)));
            if (!p)
            {
                std::fprintf(stderr, "Host memory allocation failed\n");
                std::exit(EXIT_FAILURE);
            }
            break;
        case GPU:
            CUDA_CHECK(cudaMalloc((void **)&p, n * sizeof(T)));
            break;
        }
        return p;
    }

    void zero(cudaStream_t stream)
    {
        if (devtype_ == GPU)
            CUDA_CHECK(cudaMemsetAsync(data_, 0, size_ * sizeof(T), stream));
        else
            std::memset(static_cast<void *>(data_), 0, size_ * sizeof(T));
    }

    void migrate(DeviceType to, cudaStream_t stream)
    {
        if (!data_ || devtype_ == to)
            return;
        T *p = allocate(to, size_);
        const cudaMemcpyKind kind = devtype_ == GPU ? cudaMemcpyDeviceToHost
                                    : to == GPU     ? cudaMemcpyHostToDevice
                                                    : cudaMemcpyHostToHost;
        CUDA_CHECK(cudaMemcpyAsync(p, data_, size_ * sizeof(T), kind, stream));
        CUDA_CHECK(cudaStreamSynchronize(stream));
        release();
        data_ = p;
        devtype_ = to;
    }

    void release()
    {
        if (!data_)
            return;
        switch (devtype_)
        {
        case CPU_PINNED:
            CUDA_CHECK(cudaFreeHost(data_));
            break;
        case CPU:
            std::free(data_);
            break;
        case GPU:
            CUDA_CHECK(cudaFree(data_));
            break;
        }
        data_ = nullptr;
    }

    T *data_;
};

using TensorMap = std::unordered_map<std::string, std::unique_ptr<BaseTensor>>;
