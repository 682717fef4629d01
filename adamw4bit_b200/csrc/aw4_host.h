// aw4_host.h -- host-side helpers of the C ABI: error reporting, device
// selection and the launch counter.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace aw4 {

// Records a printf-style message for aw4_last_error() (per calling thread)
// and returns `code`.
int32_t fail(int32_t code, const char* fmt, ...);

// Counts kernel launches (reported by aw4_launch_count()).
void note_launch();

// Makes `device` current for the duration of a call, restoring the caller's
// device afterwards.
class DeviceGuard {
public:
    explicit DeviceGuard(int device) : prev_(-1), ok_(true) {
        if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
        if (prev_ != device) ok_ = cudaSetDevice(device) == cudaSuccess;
        else prev_ = -1;
    }
    ~DeviceGuard() {
        if (prev_ >= 0) cudaSetDevice(prev_);
    }
    bool ok() const { return ok_; }

private:
    int prev_;
    bool ok_;
};

}  // namespace aw4
