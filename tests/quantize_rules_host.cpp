// quantize_rules_host.cpp - the library's quantization rules (csrc/quantize.cuh)
// instantiated as host code, group by group as the quantize kernel applies
// them, for test_quantize_rules.py to compare with the oracle's quantizer.
// Test infrastructure only; built with g++ by the test.
#include <cmath>
#include <cstdint>
#include <cstring>

#include "quantize.cuh"

using namespace qmm::quant;

extern "C" int qr_quantize(int mode, const float* w, int64_t n, int64_t k, uint8_t* codes, uint8_t* scales) {
    const int group = mode == 1 ? 32 : 16;
    if (k <= 0 || k % group) return -1;
    const int64_t ng = k / group, row_bytes = mode == 1 ? k : k / 2;
    for (int64_t r = 0; r < n; ++r) {
        uint8_t* cr = codes + r * row_bytes;
        std::memset(cr, 0, (size_t)row_bytes);
        for (int64_t g = 0; g < ng; ++g) {
            const float* v = w + r * k + g * group;
            float amax = 0.0f;
            for (int i = 0; i < group; ++i) amax = max_skip_nan(amax, std::fabs(v[i]));
            if (mode == 1) {
                const int x = mx_shared_exp(amax);
                const float inv = pow2f(-x);
                scales[r * ng + g] = (uint8_t)(x + 127);
                for (int i = 0; i < group; ++i) cr[g * group + i] = (uint8_t)encode_e4m3(mul_rn(v[i], inv));
            } else {
                const uint32_t sq = encode_e4m3(div_rn(amax, 6.0f));
                const float sd = e4m3_value(sq);
                scales[r * ng + g] = (uint8_t)sq;
                for (int i = 0; i < group; ++i) {
                    const int64_t kk = g * group + i;
                    cr[kk >> 1] |= (uint8_t)(nvfp4_code(v[i], sd) << ((kk & 1) * 4));
                }
            }
        }
    }
    return 0;
}
