// device_guard.cuh -- make the device that owns a stream current for the
// duration of one library call, then restore the caller's device.
//
// The library links the CUDA runtime statically, so its notion of the
// "current device" is separate from the caller's runtime (PyTorch, the
// harness).  Every entry point therefore derives the device from the stream
// it is given (or keeps the current one for the legacy default stream, and
// for a stream being captured into a CUDA graph).
#pragma once
#include <cuda_runtime.h>

struct StreamDeviceGuard {
  int prev = -1;
  int dev = 0;
  bool ok = true;
  explicit StreamDeviceGuard(cudaStream_t s) {
    if (cudaGetDevice(&prev) != cudaSuccess) { prev = -1; cudaGetLastError(); }
    dev = prev < 0 ? 0 : prev;
    // A stream being captured into a CUDA graph is not queried for its device:
    // that query invalidates the capture.  The capturing thread has the
    // stream's device current, so the current device is kept.
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (s != nullptr && cudaStreamIsCapturing(s, &cap) != cudaSuccess) { cudaGetLastError(); cap = cudaStreamCaptureStatusNone; }
    if (s != nullptr && cap == cudaStreamCaptureStatusNone) {
      int d = 0;
      if (cudaStreamGetDevice(s, &d) == cudaSuccess) {
        dev = d;
        if (d != prev && cudaSetDevice(d) != cudaSuccess) { ok = false; cudaGetLastError(); }
      } else {
        cudaGetLastError();
      }
    }
  }
  ~StreamDeviceGuard() {
    if (prev >= 0 && prev != dev) cudaSetDevice(prev);
  }
};
