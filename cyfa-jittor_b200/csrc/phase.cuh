// Clock phase of the write vector and of the readout rotations.
//
// For clock value lam and Fourier pair p (0 <= p < 64, period R = 127):
//   coord = ((floor(lam) mod 127) * p mod 127) + frac(lam) * p,
//   wrapped to (-63.5, 63.5];  phi = coord * 2*pi/127.
// The integer part is reduced exactly, so the angle stays accurate for large
// clocks.  This is the coordinate rule of cyclic_flow_attention/ops/utils.py:562-572
// (CLOCK_PHASE_HEADER :649-661) and ops/fused_recurrent.py:95-101.
#pragma once

namespace cyfa {

constexpr float kTwoPiOver127 = 0.04947390005653217f;  // 2*pi/127

__device__ __forceinline__ float clock_phase(float lam, int pair) {
  const float whole = floorf(lam);
  const float frac = lam - whole;
  int wi = static_cast<int>(whole) % 127;
  if (wi < 0) wi += 127;
  float coord = static_cast<float>((wi * pair) % 127) + frac * static_cast<float>(pair);
  if (coord > 63.5f) coord -= 127.f;
  return coord * kTwoPiOver127;
}

// Atom scale s_p of the write vector: sqrt(1/127) for pair 0, sqrt(2/127) otherwise.
__device__ __forceinline__ float atom_scale(int pair) {
  return pair == 0 ? 0.08873565094161139f : 0.12549116102763172f;
}

}  // namespace cyfa
