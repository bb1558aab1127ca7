// xspmm/core/executor.hpp -- memory/copy abstraction and the CUDA executor.
//
// Mirrors the reference's Executor / CudaExecutor (include/xspmm/core/executor.hpp:10-51,
// src/core/executor.cpp:80-108): virtual allocate / free / copy_* / synchronize, copies
// synchronous on return. CudaExecutor wraps an xspmm_b200 handle (include/xspmm_b200.h) bound to
// a device and a stream (default: the legacy default stream, as in the reference); the device is
// made current inside every call rather than only in the constructor, so executors on different
// devices can be mixed in one thread. The reference's CpuExecutor and HipExecutor are not
// provided: this library has no CPU or HIP execution path.
#pragma once

#include <cstddef>
#include <memory>
#include <stdexcept>
#include <string>

#include "../../xspmm_b200.h"

namespace xspmm {

namespace detail {
// Maps a status of the C ABI to the reference's exception types (std::invalid_argument for bad
// arguments, std::runtime_error otherwise, src/core/executor.cpp:11-19).
inline void check(xspmm_status_t s) {
    if (s == XSPMM_STATUS_OK) return;
    std::string msg = std::string("xspmm_b200: ") + xspmm_status_string(s) + ": " +
                      xspmm_last_error();
    if (s == XSPMM_STATUS_INVALID_ARGUMENT) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}
}  // namespace detail

class Executor {
public:
    virtual ~Executor() = default;
    virtual void allocate(void** ptr, size_t bytes) const = 0;
    virtual void free(void* ptr) const = 0;
    virtual void copy_from_host(void* device_dst, const void* host_src, size_t bytes) const = 0;
    virtual void copy_to_host(void* host_dst, const void* device_src, size_t bytes) const = 0;
    virtual void copy_device_to_device(void* dst, const void* src, size_t bytes) const = 0;
    virtual void synchronize() const = 0;
};

class CudaExecutor : public Executor {
public:
    explicit CudaExecutor(int device_id = 0, void* stream = nullptr) : device_id_(device_id) {
        detail::check(xspmm_create(device_id, stream, &h_));
    }
    ~CudaExecutor() override {
        if (h_) xspmm_destroy(h_);
    }
    CudaExecutor(const CudaExecutor&) = delete;
    CudaExecutor& operator=(const CudaExecutor&) = delete;

    void allocate(void** ptr, size_t bytes) const override {
        detail::check(xspmm_malloc(h_, ptr, bytes));
    }
    void free(void* ptr) const override { detail::check(xspmm_free(h_, ptr)); }
    void copy_from_host(void* dst, const void* src, size_t bytes) const override {
        detail::check(xspmm_memcpy_h2d(h_, dst, src, bytes));
    }
    void copy_to_host(void* dst, const void* src, size_t bytes) const override {
        detail::check(xspmm_memcpy_d2h(h_, dst, src, bytes));
    }
    void copy_device_to_device(void* dst, const void* src, size_t bytes) const override {
        detail::check(xspmm_memcpy_d2d(h_, dst, src, bytes));
    }
    void synchronize() const override { detail::check(xspmm_synchronize(h_)); }

    void set_stream(void* stream) const { detail::check(xspmm_set_stream(h_, stream)); }
    int device_id() const { return device_id_; }
    xspmm_handle_t handle() const { return h_; }

private:
    int device_id_;
    xspmm_handle_t h_ = nullptr;
};

namespace detail {
inline xspmm_handle_t handle_of(const std::shared_ptr<const Executor>& exec) {
    auto* c = dynamic_cast<const CudaExecutor*>(exec.get());
    if (!c) throw std::runtime_error("xspmm_b200 runs on a CudaExecutor only");
    return c->handle();
}
}  // namespace detail

}  // namespace xspmm
