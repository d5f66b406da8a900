/*
 * TEST INFRASTRUCTURE ONLY -- builds the reference's own onboard
 * tactical/prior device header (src/network/onboard_features.cuh:1-521) as
 * host C++ so that its outputs can serve as the CPU oracle for the onboard
 * kernel.  The header is compiled from where it lies in the reference tree
 * (include path given by oracle/Makefile); nothing of it is copied here.
 * The output goes to oracle/_ref/, which is never committed.
 */
#include <cmath>
#include <math.h>

using std::isinf;
using std::isnan;

#define __device__
#define __forceinline__ inline
#include "onboard_features.cuh"

extern "C" void tb_ref_onboard_tactical_prior(const float *obs_4148, const float *mission_10,
                                              float *tactical_24, float *prior_15) {
    tb_onboard_tactical_prior(obs_4148, mission_10, tactical_24, prior_15);
}

extern "C" void tb_ref_onboard_batch(const float *obs, const float *mission, size_t count,
                                     float *out_39) {
    for (size_t i = 0; i < count; ++i)
        tb_onboard_tactical_prior(obs + i * 4148, mission + i * 10, out_39 + i * 39,
                                  out_39 + i * 39 + 24);
}
