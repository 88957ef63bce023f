// Host-built RoPE tables (cos, sin per position and rotated pair) with ggml's NEOX cache
// arithmetic: theta_i = p * theta_scale^i by repeated f32 multiplication, theta_scale =
// powf(base, -2/hd), divided by an optional per-pair frequency factor and scaled by freq_scale
// (ext_factor 0, attn_factor 1).
#pragma once

#include <cmath>
#include <vector>
#include <vector_types.h>

namespace bzb {

inline std::vector<float2> rope_table(int max_pos, int hd, float base, float fscale, const std::vector<float> * ff) {
    const int half = hd / 2;
    const float ts = powf(base, -2.0f / (float) hd);
    std::vector<float2> tab((size_t) max_pos * half);
    for (int p = 0; p < max_pos; p++) {
        float theta = (float) p;
        for (int i = 0; i < half; i++) {
            float t = ff ? theta / (*ff)[i] : theta;
            t = fscale * t;
            tab[(size_t) p * half + i] = make_float2(cosf(t), sinf(t));
            theta *= ts;
        }
    }
    return tab;
}

}  // namespace bzb
