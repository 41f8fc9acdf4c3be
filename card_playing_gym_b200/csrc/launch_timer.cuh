// CUDA-event timing of one family of kernel launches (a measurement hook, off by default):
// while enabled, each launch is bracketed by a pair of events on its stream.
#pragma once

#include "common.cuh"

namespace cg {

struct LaunchTimer {
  bool enabled = false;
  int capacity = 0;
  int count = 0;
  cudaEvent_t* start = nullptr;
  cudaEvent_t* stop = nullptr;

  // Enabling clears earlier records and makes room for `capacity` launches.
  int configure(int enable, int new_capacity, const char* who) {
    for (int i = 0; i < capacity; ++i) {
      cudaEventDestroy(start[i]);
      cudaEventDestroy(stop[i]);
    }
    delete[] start;
    delete[] stop;
    enabled = false;
    capacity = count = 0;
    start = stop = nullptr;
    if (!enable) return CG_OK;
    CG_REQUIRE(new_capacity > 0 && new_capacity <= (1 << 20), "%s: capacity 1..2^20", who);
    start = new cudaEvent_t[new_capacity];
    stop = new cudaEvent_t[new_capacity];
    for (int i = 0; i < new_capacity; ++i) {
      if (cudaEventCreate(&start[i]) != cudaSuccess) return set_error(CG_ERR_CUDA, "%s: cudaEventCreate failed", who);
      if (cudaEventCreate(&stop[i]) != cudaSuccess) {
        cudaEventDestroy(start[i]);
        return set_error(CG_ERR_CUDA, "%s: cudaEventCreate failed", who);
      }
      capacity = i + 1;
    }
    enabled = true;
    return CG_OK;
  }

  // Synchronizes; writes up to max_count durations in milliseconds; returns how many (or -1).
  int timings(float* ms_out, int max_count) {
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    const int n = count < max_count ? count : max_count;
    for (int i = 0; i < n; ++i)
      if (cudaEventElapsedTime(&ms_out[i], start[i], stop[i]) != cudaSuccess) return -1;
    return n;
  }

  bool begin(cudaStream_t s) {
    const bool record = enabled && count < capacity;
    if (record) cudaEventRecord(start[count], s);
    return record;
  }

  void end(cudaStream_t s, bool recorded) {
    if (recorded) cudaEventRecord(stop[count++], s);
  }
};

}  // namespace cg
