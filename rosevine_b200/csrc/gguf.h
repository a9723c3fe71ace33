// gguf.h - a GGUF v3 reader for the MoE layer's weights (host code of librvcuda.so).
//
// Restates the checks of the reference's parser (runtime/src/gguf.rs:272-383, Gguf::parse) so
// that a file the reference rejects is rejected here with the same reason, and binds tensors by
// name as runtime/src/model.rs:61-107 does (Weights::bind): a tensor is a view into the file's
// mapping, nothing is copied. Only the tensor types the target uses are accepted (F32, Q4_0,
// gguf.rs:21-40). The MoE layer is then built from blk.<l>.ffn_gate_up_exps.weight /
// ffn_down_exps.weight (rvc_pack_experts input, GGUF layout), ffn_gate_inp.weight (F32 router),
// ffn_down_exps.scale and the branch's norm weights.
#pragma once
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

namespace rvc {
namespace gguf {

constexpr uint64_t kMaxKv = 65536, kMaxTensors = 65536, kMaxArrayLen = 4194304, kMaxStringLen = 16ull << 20;
constexpr uint32_t kMaxAlignment = 1u << 20, kDefaultAlignment = 32;

// Reasons, in the words of the reference's Error::Malformed strings; rvc_error_string returns
// them for RVC_ERR_GGUF + index.
enum Reason : int {
    kOk = 0,
    kTruncated,           // "truncated header"
    kBadMagic,            // "bad magic"
    kVersion,             // "expected GGUF version 3"
    kCountLimit,          // "descriptor count limit exceeded"
    kEmptyKey,            // "empty metadata key"
    kDupKey,              // "duplicate metadata key"
    kAlignment,           // "invalid alignment"
    kBool,                // "invalid bool"
    kArrayElem,           // "unsupported array element type"
    kArrayLen,            // "array length limit exceeded"
    kStringLen,           // "string length limit exceeded"
    kUtf8,                // "string is not UTF-8"
    kMetaType,            // "unsupported metadata type"
    kTensorName,          // "empty or duplicate tensor name"
    kRank,                // "invalid tensor rank"
    kType,                // "unsupported tensor type"
    kShape,               // "invalid tensor shape"
    kElemOverflow,        // "tensor element count overflow"
    kSizeOverflow,        // "tensor size overflow"
    kMisaligned,          // "misaligned tensor offset"
    kLenOverflow,         // "length overflow"
    kNoData,              // "truncated before data section"
    kRangeOverflow,       // "tensor range overflow"
    kRange,               // "overlapping or out-of-file tensor range"
    kMissing,             // "missing tensor"
    kContract,            // "tensor shape or type differs from the layer's contract"
    kIo,                  // "cannot open or map the file"
    kReasons
};
inline const char *reason(int r) {
    static const char *s[kReasons] = {"ok",
                                      "truncated header",
                                      "bad magic",
                                      "expected GGUF version 3",
                                      "descriptor count limit exceeded",
                                      "empty metadata key",
                                      "duplicate metadata key",
                                      "invalid alignment",
                                      "invalid bool",
                                      "unsupported array element type",
                                      "array length limit exceeded",
                                      "string length limit exceeded",
                                      "string is not UTF-8",
                                      "unsupported metadata type",
                                      "empty or duplicate tensor name",
                                      "invalid tensor rank",
                                      "unsupported tensor type",
                                      "invalid tensor shape",
                                      "tensor element count overflow",
                                      "tensor size overflow",
                                      "misaligned tensor offset",
                                      "length overflow",
                                      "truncated before data section",
                                      "tensor range overflow",
                                      "overlapping or out-of-file tensor range",
                                      "missing tensor",
                                      "tensor shape or type differs from the layer's contract",
                                      "cannot open or map the file"};
    return r >= 0 && r < kReasons ? s[r] : "unknown GGUF error";
}

constexpr int kF32 = 0, kQ4_0 = 2;  // GGML type ids

struct Tensor {
    std::string name;
    int dtype = 0;
    int n_dims = 0;
    uint64_t shape[4] = {1, 1, 1, 1};
    uint64_t offset = 0, bytes = 0;
    const uint8_t *data = nullptr;
};

struct File {
    const uint8_t *buf = nullptr;
    size_t len = 0;
    void *map = nullptr;  // the mapping this object owns (rvc_gguf_open), else null
    size_t map_len = 0;
    uint32_t alignment = kDefaultAlignment;
    uint64_t data_offset = 0;
    std::string arch;  // general.architecture, if a string
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, size_t> index;

    const Tensor *find(const char *name) const {
        auto it = index.find(name);
        return it == index.end() ? nullptr : &tensors[it->second];
    }
};

// Strict UTF-8 (no overlongs, surrogates or code points above U+10FFFF), as Rust's str.
inline bool utf8_ok(const uint8_t *p, uint64_t n) {
    uint64_t i = 0;
    while (i < n) {
        const uint8_t c = p[i];
        int k;
        uint32_t cp;
        if (c < 0x80) {
            ++i;
            continue;
        } else if ((c & 0xE0) == 0xC0) {
            k = 1, cp = c & 0x1F;
        } else if ((c & 0xF0) == 0xE0) {
            k = 2, cp = c & 0x0F;
        } else if ((c & 0xF8) == 0xF0) {
            k = 3, cp = c & 0x07;
        } else {
            return false;
        }
        if (n - i <= (uint64_t)k) return false;  // the sequence runs past the end
        for (int j = 1; j <= k; ++j) {
            if ((p[i + j] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (p[i + j] & 0x3F);
        }
        if ((k == 1 && cp < 0x80) || (k == 2 && cp < 0x800) || (k == 3 && cp < 0x10000) || cp > 0x10FFFF ||
            (cp >= 0xD800 && cp <= 0xDFFF))
            return false;
        i += k + 1;
    }
    return true;
}

struct Cursor {
    const uint8_t *buf;
    uint64_t len, pos = 0;
    int err = kOk;
    bool take(uint64_t n, const uint8_t **p) {
        if (err) return false;
        if (n > len - pos) return fail(kTruncated);
        *p = buf + pos;
        pos += n;
        return true;
    }
    bool fail(int r) {
        if (!err) err = r;
        return false;
    }
    bool u32(uint32_t *v) {
        const uint8_t *p;
        if (!take(4, &p)) return false;
        std::memcpy(v, p, 4);
        return true;
    }
    bool u64(uint64_t *v) {
        const uint8_t *p;
        if (!take(8, &p)) return false;
        std::memcpy(v, p, 8);
        return true;
    }
    bool str(std::string *s) {
        uint64_t n;
        if (!u64(&n)) return false;
        if (n > kMaxStringLen) return fail(kStringLen);
        const uint8_t *p;
        if (!take(n, &p)) return false;
        if (!utf8_ok(p, n)) return fail(kUtf8);
        if (s) s->assign(reinterpret_cast<const char *>(p), n);
        return true;
    }
    // Scalar sizes of the metadata types 0..7, 10..12 (gguf.rs:59-83); 0 for the others.
    static int scalar_size(uint32_t t) {
        switch (t) {
            case 0: case 1: case 7: return 1;
            case 2: case 3: return 2;
            case 4: case 5: case 6: return 4;
            case 10: case 11: case 12: return 8;
            default: return 0;
        }
    }
    // One metadata value; a string value is returned through `s` when asked for.
    bool value(uint32_t type, std::string *s) {
        if (const int sz = scalar_size(type)) {
            const uint8_t *p;
            if (!take((uint64_t)sz, &p)) return false;
            if (type == 7 && p[0] > 1) return fail(kBool);
            return true;
        }
        if (type == 8) return str(s);
        if (type != 9) return fail(kMetaType);
        uint32_t elem;
        uint64_t count;
        if (!u32(&elem) || !u64(&count)) return false;
        if (count > kMaxArrayLen) return fail(kArrayLen);
        if (const int sz = scalar_size(elem)) {
            const uint8_t *p;
            if (!take(count * (uint64_t)sz, &p)) return false;
            if (elem == 7)
                for (uint64_t i = 0; i < count; ++i)
                    if (p[i] > 1) return fail(kBool);
            return true;
        }
        if (elem != 8) return fail(kArrayElem);
        if (count > (len - pos) / 8) return fail(kTruncated);  // each string needs its 8-byte length
        for (uint64_t i = 0; i < count; ++i)
            if (!str(nullptr)) return false;
        return true;
    }
};

// Parse and validate `buf` (the whole file); tensors become views into it.
inline int parse(const uint8_t *buf, size_t len, File *f) {
    Cursor c{buf, (uint64_t)len};
    const uint8_t *magic;
    if (!c.take(4, &magic)) return c.err;
    if (std::memcmp(magic, "GGUF", 4) != 0) return kBadMagic;
    uint32_t version;
    uint64_t n_tensors, n_kv;
    if (!c.u32(&version)) return c.err;
    if (version != 3) return kVersion;
    if (!c.u64(&n_tensors) || !c.u64(&n_kv)) return c.err;
    if (n_tensors == 0 || n_tensors > kMaxTensors || n_kv > kMaxKv) return kCountLimit;
    std::unordered_map<std::string, int> keys;
    bool have_align = false;
    uint64_t align_v = 0;
    bool align_int = false;
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key, sval;
        uint32_t type;
        if (!c.str(&key) || !c.u32(&type)) return c.err;
        if (key.empty()) return kEmptyKey;
        const uint64_t vpos = c.pos;
        if (!c.value(type, &sval)) return c.err;
        if (!keys.emplace(key, 1).second) return kDupKey;
        if (key == "general.alignment") {
            have_align = true;
            const int sz = Cursor::scalar_size(type);
            align_int = sz && type != 6 && type != 7 && type != 12;  // an integer type
            if (align_int) {
                int64_t v = 0;
                uint64_t u = 0;
                std::memcpy(&u, buf + vpos, (size_t)sz);
                const bool sgn = type == 1 || type == 3 || type == 5 || type == 11;
                if (sgn) {  // sign-extend
                    const int bits = 8 * sz;
                    v = bits == 64 ? (int64_t)u : (int64_t)(u << (64 - bits)) >> (64 - bits);
                    align_int = v >= 0;
                    u = (uint64_t)v;
                }
                align_v = u;
            }
        }
        if (key == "general.architecture" && type == 8) f->arch = sval;
    }
    f->alignment = kDefaultAlignment;
    if (have_align) {
        if (!align_int || align_v < 1 || align_v > kMaxAlignment || (align_v & (align_v - 1))) return kAlignment;
        f->alignment = (uint32_t)align_v;
    }
    f->tensors.clear();
    f->index.clear();
    for (uint64_t i = 0; i < n_tensors; ++i) {
        Tensor t;
        uint32_t n_dims, type;
        if (!c.str(&t.name)) return c.err;
        if (t.name.empty() || !f->index.emplace(t.name, (size_t)i).second) return kTensorName;
        if (!c.u32(&n_dims)) return c.err;
        if (n_dims < 1 || n_dims > 4) return kRank;
        t.n_dims = (int)n_dims;
        for (uint32_t d = 0; d < n_dims; ++d)
            if (!c.u64(&t.shape[d])) return c.err;
        if (!c.u32(&type)) return c.err;
        if (type != kF32 && type != kQ4_0) return kType;
        t.dtype = (int)type;
        if (!c.u64(&t.offset)) return c.err;
        const uint64_t block = type == kQ4_0 ? 32 : 1, block_bytes = type == kQ4_0 ? 18 : 4;
        for (uint32_t d = 0; d < n_dims; ++d)
            if (t.shape[d] == 0) return kShape;
        if (t.shape[0] % block) return kShape;
        uint64_t elems = 1;
        for (uint32_t d = 0; d < n_dims; ++d) {
            if (t.shape[d] && elems > UINT64_MAX / t.shape[d]) return kElemOverflow;
            elems *= t.shape[d];
        }
        if (elems >= (1ull << 62)) return kElemOverflow;
        if (elems / block > UINT64_MAX / block_bytes) return kSizeOverflow;
        t.bytes = elems / block * block_bytes;
        if (t.offset % f->alignment) return kMisaligned;
        f->tensors.push_back(std::move(t));
    }
    const uint64_t a = f->alignment;
    if (c.pos > UINT64_MAX - (a - 1)) return kLenOverflow;
    f->data_offset = (c.pos + a - 1) / a * a;
    if (f->data_offset > len) return kNoData;
    std::vector<size_t> order(f->tensors.size());
    for (size_t i = 0; i < order.size(); ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(),
                     [&](size_t x, size_t y) { return f->tensors[x].offset < f->tensors[y].offset; });
    uint64_t end = 0;
    for (size_t i : order) {
        const Tensor &t = f->tensors[i];
        if (t.offset > UINT64_MAX - t.bytes) return kRangeOverflow;
        const uint64_t stop = t.offset + t.bytes;
        if (t.offset < end || f->data_offset > UINT64_MAX - stop || f->data_offset + stop > len) return kRange;
        end = stop;
    }
    for (Tensor &t : f->tensors) t.data = buf + f->data_offset + t.offset;
    f->buf = buf, f->len = len;
    return kOk;
}

}  // namespace gguf
}  // namespace rvc
