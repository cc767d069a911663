// spec.cpp - quantization-spec inference and argument resolution (pure host).
//
// qmm_infer_quant_spec restates inferQuantSpec (src/weights.zig:132-185)
// rule for rule, including its error classes and the order in which they
// are checked, so a checkpoint that loads (or fails) in the reference loads
// (or fails the same way) here.
#include <cstring>
#include <string>

#include "internal.h"

namespace {

// src/weights.zig:136: pbuf is 1024 bytes; "<prefix>.weight" must fit.
constexpr size_t kNameBuf = 1024;

bool ends_with(const char* s, const char* suf) {
    const size_t n = std::strlen(s), m = std::strlen(suf);
    return n >= m && std::memcmp(s + n - m, suf, m) == 0;
}

const qmm_tensor_info* find_info(const qmm_tensor_info* infos, int64_t count, const std::string& name) {
    for (int64_t i = 0; i < count; ++i)
        if (infos[i].name && name == infos[i].name) return &infos[i];
    return nullptr;
}

// bufPrint("{s}.weight") into the 1024-byte buffer; false on overflow.
bool sibling(const char* name, size_t strip, const char* suffix, std::string* out) {
    const size_t plen = std::strlen(name) - strip;
    if (plen + std::strlen(suffix) > kNameBuf) return false;
    out->assign(name, plen);
    out->append(suffix);
    return true;
}

}  // namespace

namespace qmm {

int check_spec(const qmm_quant_spec& s) {
    if (s.mode == QMM_MODE_MXFP8 && s.group_size == 32 && s.bits == 8) return QMM_OK;
    if (s.mode == QMM_MODE_NVFP4 && s.group_size == 16 && s.bits == 4) return QMM_OK;
    return set_error(QMM_ERR_BAD_MODE, "unsupported quantization (mode=%d, group=%d, bits=%d): "
                     "only mxfp8 (32, 8) and nvfp4 (16, 4)", s.mode, s.group_size, s.bits);
}

}  // namespace qmm

extern "C" int qmm_infer_quant_spec(const qmm_tensor_info* infos, int64_t count, qmm_quant_spec* out) {
    using qmm::set_error;
    if (!out || (count > 0 && !infos) || count < 0)
        return set_error(QMM_ERR_BAD_ARGUMENT, "qmm_infer_quant_spec: null argument");
    for (int64_t i = 0; i < count; ++i)
        if (!infos[i].name || (infos[i].ndim > 0 && !infos[i].shape) || infos[i].ndim < 0)
            return set_error(QMM_ERR_BAD_ARGUMENT, "qmm_infer_quant_spec: tensor %lld malformed", (long long)i);
    *out = qmm_quant_spec{QMM_MODE_NONE, 0, 0};

    // weights.zig:133-145: the first "*.scales" decides; none -> dense unless
    // a packed U32/U8 tensor exists.
    const qmm_tensor_info* sc = nullptr;
    for (int64_t i = 0; i < count; ++i)
        if (ends_with(infos[i].name, ".scales")) { sc = &infos[i]; break; }
    if (!sc) {
        for (int64_t i = 0; i < count; ++i)
            if (infos[i].dtype == QMM_DTYPE_U32 || infos[i].dtype == QMM_DTYPE_U8)
                return set_error(QMM_ERR_NONSTANDARD_QUANT, "packed tensor '%s' without any *.scales", infos[i].name);
        return QMM_OK;
    }
    // weights.zig:146-147
    if (sc->ndim != 2) return set_error(QMM_ERR_NONSTANDARD_QUANT, "'%s' is not 2-D", sc->name);
    if (sc->dtype != QMM_DTYPE_U8)
        return set_error(QMM_ERR_AFFINE_UNSUPPORTED, "'%s' is not U8 (affine quantization is unsupported)", sc->name);
    // weights.zig:149-156: sibling "<prefix>.weight" U32 [out, packed]
    const size_t sl = std::strlen(".scales");
    std::string wname;
    if (std::strlen(sc->name) < sl + 1 || !sibling(sc->name, sl, ".weight", &wname))
        return set_error(QMM_ERR_NONSTANDARD_QUANT, "bad scales name '%s'", sc->name);
    const qmm_tensor_info* w = find_info(infos, count, wname);
    if (!w) return set_error(QMM_ERR_NONSTANDARD_QUANT, "'%s' has no packed '%s'", sc->name, wname.c_str());
    if (w->dtype != QMM_DTYPE_U32 || w->ndim != 2)
        return set_error(QMM_ERR_NONSTANDARD_QUANT, "'%s' is not a 2-D U32 tensor", wname.c_str());
    // weights.zig:157-166: r = packed_cols / scale_cols
    const int64_t packed_d1 = w->shape[1], sgroups = sc->shape[1];
    if (packed_d1 <= 0 || sgroups <= 0 || packed_d1 % sgroups != 0)
        return set_error(QMM_ERR_NONSTANDARD_QUANT, "packed cols %lld not a multiple of scale cols %lld",
                         (long long)packed_d1, (long long)sgroups);
    const int64_t r = packed_d1 / sgroups;
    qmm_quant_spec spec;
    if (r == 8) spec = qmm_quant_spec{QMM_MODE_MXFP8, 32, 8};
    else if (r == 2) spec = qmm_quant_spec{QMM_MODE_NVFP4, 16, 4};
    else return set_error(QMM_ERR_NONSTANDARD_QUANT, "packed/scales ratio %lld is neither 8 nor 2", (long long)r);
    // weights.zig:167-183: every scales tensor agrees, no orphan packed weight.
    const size_t wl = std::strlen(".weight");
    for (int64_t i = 0; i < count; ++i) {
        const qmm_tensor_info& t = infos[i];
        if (ends_with(t.name, ".scales")) {
            if (t.dtype != QMM_DTYPE_U8 || t.ndim != 2)
                return set_error(QMM_ERR_INCONSISTENT_QUANT, "'%s' is not a 2-D U8 tensor", t.name);
            std::string wn;
            if (!sibling(t.name, sl, ".weight", &wn))
                return set_error(QMM_ERR_NONSTANDARD_QUANT, "bad scales name '%s'", t.name);
            const qmm_tensor_info* w2 = find_info(infos, count, wn);
            if (!w2) return set_error(QMM_ERR_NONSTANDARD_QUANT, "'%s' has no packed '%s'", t.name, wn.c_str());
            if (w2->dtype != QMM_DTYPE_U32 || w2->ndim != 2)
                return set_error(QMM_ERR_NONSTANDARD_QUANT, "'%s' is not a 2-D U32 tensor", wn.c_str());
            const int64_t p2 = w2->shape[1];
            if (t.shape[1] <= 0 || p2 % t.shape[1] != 0 || p2 / t.shape[1] != r)
                return set_error(QMM_ERR_INCONSISTENT_QUANT, "'%s' ratio differs from the checkpoint's %lld",
                                 t.name, (long long)r);
        }
        if (t.dtype == QMM_DTYPE_U32 && ends_with(t.name, ".weight")) {
            std::string sn;
            if (!sibling(t.name, wl, ".scales", &sn))
                return set_error(QMM_ERR_NONSTANDARD_QUANT, "bad weight name '%s'", t.name);
            if (!find_info(infos, count, sn))
                return set_error(QMM_ERR_INCONSISTENT_QUANT, "packed '%s' has no scales", t.name);
        }
    }
    *out = spec;
    return QMM_OK;
}

extern "C" const char* qmm_mode_str(qmm_quant_spec spec) {
    // src/weights.zig:47-53: .none maps to "mxfp8" and is never used for a qmm.
    return spec.mode == QMM_MODE_NVFP4 ? "nvfp4" : "mxfp8";
}

extern "C" int qmm_spec_from_args(qmm_optional_int group_size, qmm_optional_int bits, const char* mode,
                                  qmm_quant_spec* out) {
    using qmm::set_error;
    if (!mode || !out) return set_error(QMM_ERR_BAD_ARGUMENT, "qmm_spec_from_args: null mode or out");
    qmm_quant_spec s;
    if (std::strcmp(mode, "mxfp8") == 0) s = qmm_quant_spec{QMM_MODE_MXFP8, 32, 8};
    else if (std::strcmp(mode, "nvfp4") == 0) s = qmm_quant_spec{QMM_MODE_NVFP4, 16, 4};
    else return set_error(QMM_ERR_BAD_MODE, "mode '%s' is not supported (mxfp8, nvfp4)", mode);
    if (group_size.has_value && group_size.value != s.group_size)
        return set_error(QMM_ERR_BAD_MODE, "%s requires group_size %d, got %d", mode, s.group_size, group_size.value);
    if (bits.has_value && bits.value != s.bits)
        return set_error(QMM_ERR_BAD_MODE, "%s requires bits %d, got %d", mode, s.bits, bits.value);
    *out = s;
    return QMM_OK;
}
