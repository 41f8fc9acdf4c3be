// The device half of the PPO baseline: per-decision seat values and the zero-sum projection.
//
// References: cardgym/rl/trainer.py:556-571 (the critic's seat-value gather: absolute seat i sits at
// column (i - shift) mod players of the stream's values, inactive seats zero, the acting seat's
// entry is the decision's prediction), trainer.py:610-632 (_recorded_values: the rollout-recorded
// values centred over the active seats in float64, acting seat first), cardgym/rl/ppo.py:97-108
// (center_zero_sum: subtract the active seats' mean, zero the padded seats).
//
// Row and seat indices are checked on the device: a row outside the values or a player count
// outside [1, seats] writes zeros for that decision and sets the fault word (0x400 / 0x401).
#include "common.cuh"

namespace cg {

constexpr int kMaxSeats = 8;

// One thread per decision. values f32 [value_rows, seats]; the decision reads row flat[i] (or i).
// center = 0: the values are already centred (the critic's pending values); prediction = the
//             acting seat's gathered value, state[i, s] = values[row, (s - shift) mod players].
// center = 1: the values are raw recorded values: centred here in float64 (sequential sum over all
//             columns from 0, the numpy order for rows shorter than 8), prediction = centred column 0
//             (the acting seat first), state gathered from the centred row.
__global__ void seat_values_kernel(const float* __restrict__ values, int64_t value_rows, int seats,
                                   const int64_t* __restrict__ flat, const int64_t* __restrict__ shift,
                                   const int64_t* __restrict__ players, const int64_t* __restrict__ seat, int64_t n,
                                   int center, double* __restrict__ state, double* __restrict__ prediction) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t row = flat ? flat[i] : i;
  const int64_t count = players[i];
  const int64_t acting = seat[i];
  double out[kMaxSeats];
  double pred = 0.0;
#pragma unroll
  for (int s = 0; s < kMaxSeats; ++s) out[s] = 0.0;
  const bool row_ok = row >= 0 && row < value_rows;
  const bool count_ok = count >= 1 && count <= seats;
  if (!row_ok) raise_fault(0x400);
  if (!count_ok) raise_fault(0x401);
  if (row_ok && count_ok) {
    double v[kMaxSeats];
#pragma unroll
    for (int s = 0; s < kMaxSeats; ++s) v[s] = s < seats ? static_cast<double>(values[row * seats + s]) : 0.0;
    if (center) {
      double total = 0.0;
#pragma unroll
      for (int s = 0; s < kMaxSeats; ++s)
        if (s < seats) {
          v[s] = s < count ? v[s] : 0.0;
          total = __dadd_rn(total, v[s]);
        }
      const double mean = __ddiv_rn(total, static_cast<double>(count));
#pragma unroll
      for (int s = 0; s < kMaxSeats; ++s) v[s] = s < count ? __dsub_rn(v[s], mean) : 0.0;
      pred = v[0];
    }
    const int64_t rot = ((-shift[i]) % count + count) % count;  // column of seat s: (s + rot) mod count
#pragma unroll
    for (int s = 0; s < kMaxSeats; ++s)
      if (s < count) out[s] = v[(s + rot) % count];
    if (!center) pred = (acting >= 0 && acting < count) ? out[acting] : 0.0;
  }
  if (state) {
#pragma unroll
    for (int s = 0; s < kMaxSeats; ++s)
      if (s < seats) state[i * seats + s] = out[s];
  }
  if (prediction) prediction[i] = pred;
}

// center_zero_sum (ppo.py:97-108) in float32: mean = (sum over active seats) / players, in seat order.
__global__ void center_zero_sum_kernel(const float* __restrict__ values, const int64_t* __restrict__ players,
                                       int64_t n, int seats, float* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int64_t count = players[i];
  float total = 0.f;
  for (int s = 0; s < seats; ++s) total = __fadd_rn(total, s < count ? values[i * seats + s] : 0.f);
  const float mean = __fdiv_rn(total, static_cast<float>(count));
  for (int s = 0; s < seats; ++s) out[i * seats + s] = s < count ? __fsub_rn(values[i * seats + s], mean) : 0.f;
}

}  // namespace cg

extern "C" int cg_seat_values(const float* values, int64_t value_rows, int seats, const int64_t* flat,
                              const int64_t* shift, const int64_t* players, const int64_t* seat, int64_t n, int center,
                              double* state_out, double* prediction_out, void* stream) {
  using namespace cg;
  CG_REQUIRE(seats >= 1 && seats <= kMaxSeats, "cg_seat_values: seats must be 1..%d", kMaxSeats);
  CG_REQUIRE(n >= 0 && value_rows >= 0 && (center == 0 || center == 1), "cg_seat_values: bad arguments");
  if (n == 0) return CG_OK;
  CG_REQUIRE(values && shift && players && seat && (state_out || prediction_out), "cg_seat_values: NULL pointer");
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
  seat_values_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      values, value_rows, seats, flat, shift, players, seat, n, center, state_out, prediction_out);
  return check_launch("seat_values_kernel");
}

extern "C" int cg_center_zero_sum(const float* values, const int64_t* players, int64_t n, int seats, float* out,
                                  void* stream) {
  using namespace cg;
  CG_REQUIRE(seats >= 1 && n >= 0, "cg_center_zero_sum: bad shape");
  if (n == 0) return CG_OK;
  CG_REQUIRE(values && players && out, "cg_center_zero_sum: NULL pointer");
  const unsigned blocks = static_cast<unsigned>((n + 255) / 256);
  center_zero_sum_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(values, players, n, seats, out);
  return check_launch("center_zero_sum_kernel");
}
