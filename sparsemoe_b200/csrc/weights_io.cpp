// Expert weight files (.bin): one layer's router and expert weights, in the
// formats the kernels read directly (16-bit, int8 with per-tensor or
// per-channel scales, FP8 with 128x128 block scales, pair-interleaved 4-bit
// nibbles with INT4 scale/zero or NVFP4 scale/global arrays), so loading is a
// plain copy with no repacking.  The reference's driver has a cache-file hook
// (drivers/main.cu:27-31, ".cache/ref_N%d.bin") that nothing writes; this is
// the format the layer's weights are stored in instead.
//
// File: the MoeWeightFile header (magic "SMOEW001", format, shape, up to
// MOE_WFILE_MAX_ARRAYS array descriptors: name, element size, shape, byte
// offset and size), then each array's bytes at a 256-byte aligned offset.
// Little-endian, as the header struct lies in memory on x86-64 / aarch64.
#include <cstdint>
#include <cstdio>
#include <cstring>

#include "../../include/sparsemoe_b200.h"

namespace {

constexpr char kMagic[8] = {'S', 'M', 'O', 'E', 'W', '0', '0', '1'};

uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

uint64_t elems(const MoeWeightArray& a) {
    uint64_t n = 1;
    for (int i = 0; i < a.ndim; ++i) n *= (uint64_t)a.shape[i];
    return n;
}

bool array_ok(const MoeWeightArray& a) {
    if (a.name[0] == 0 || std::memchr(a.name, 0, sizeof(a.name)) == nullptr) return false;
    if (a.elem_bytes != 1 && a.elem_bytes != 2 && a.elem_bytes != 4) return false;
    if (a.kind < 0 || a.kind > 2 || (a.kind == 2 && a.elem_bytes != 4)) return false;
    if (a.ndim < 1 || a.ndim > 4) return false;
    for (int i = 0; i < a.ndim; ++i)
        if (a.shape[i] < 0) return false;
    return true;
}

struct File {
    FILE* f = nullptr;
    explicit File(FILE* p) : f(p) {}
    ~File() {
        if (f) std::fclose(f);
    }
};

}  // namespace

extern "C" int moe_weights_write(const char* path, const MoeWeightFile* header, const void* const* data) {
    if (!path || !header || !data || header->num_arrays < 1 || header->num_arrays > MOE_WFILE_MAX_ARRAYS)
        return MOE_ERR_INVALID_ARG;
    MoeWeightFile h = *header;
    std::memcpy(h.magic, kMagic, sizeof(kMagic));
    uint64_t off = align256(sizeof(MoeWeightFile));
    for (int i = 0; i < h.num_arrays; ++i) {
        MoeWeightArray& a = h.arrays[i];
        if (!array_ok(a) || !data[i]) return MOE_ERR_INVALID_ARG;
        a.bytes = elems(a) * (uint64_t)a.elem_bytes;
        a.offset = off;
        off = align256(off + a.bytes);
    }
    File out(std::fopen(path, "wb"));
    if (!out.f) return MOE_ERR_INVALID_ARG;
    if (std::fwrite(&h, sizeof(h), 1, out.f) != 1) return MOE_ERR_INVALID_ARG;
    static const char zeros[256] = {};
    uint64_t pos = sizeof(h);
    for (int i = 0; i < h.num_arrays; ++i) {
        const MoeWeightArray& a = h.arrays[i];
        if (a.offset > pos && std::fwrite(zeros, 1, a.offset - pos, out.f) != a.offset - pos) return MOE_ERR_INVALID_ARG;
        if (a.bytes && std::fwrite(data[i], 1, a.bytes, out.f) != a.bytes) return MOE_ERR_INVALID_ARG;
        pos = a.offset + a.bytes;
    }
    return std::fflush(out.f) == 0 ? MOE_OK : MOE_ERR_INVALID_ARG;
}

extern "C" int moe_weights_read_header(const char* path, MoeWeightFile* header) {
    if (!path || !header) return MOE_ERR_INVALID_ARG;
    File in(std::fopen(path, "rb"));
    if (!in.f) return MOE_ERR_INVALID_ARG;
    MoeWeightFile h;
    if (std::fread(&h, sizeof(h), 1, in.f) != 1) return MOE_ERR_INVALID_ARG;
    if (std::memcmp(h.magic, kMagic, sizeof(kMagic)) != 0) return MOE_ERR_INVALID_ARG;
    if (h.num_arrays < 1 || h.num_arrays > MOE_WFILE_MAX_ARRAYS) return MOE_ERR_INVALID_ARG;
    if (std::fseek(in.f, 0, SEEK_END) != 0) return MOE_ERR_INVALID_ARG;
    const long size = std::ftell(in.f);
    if (size < 0) return MOE_ERR_INVALID_ARG;
    for (int i = 0; i < h.num_arrays; ++i) {
        const MoeWeightArray& a = h.arrays[i];
        if (!array_ok(a) || a.bytes != elems(a) * (uint64_t)a.elem_bytes || a.offset % 256 != 0 ||
            a.offset < sizeof(h) || a.offset + a.bytes > (uint64_t)size)
            return MOE_ERR_INVALID_ARG;   // damaged or truncated file
    }
    *header = h;
    return MOE_OK;
}

extern "C" int moe_weights_read_array(const char* path, const MoeWeightFile* header, int index, void* dst,
                                      size_t dst_bytes) {
    if (!path || !header || !dst || index < 0 || index >= header->num_arrays) return MOE_ERR_INVALID_ARG;
    const MoeWeightArray& a = header->arrays[index];
    if (dst_bytes < a.bytes) return MOE_ERR_INVALID_ARG;
    File in(std::fopen(path, "rb"));
    if (!in.f) return MOE_ERR_INVALID_ARG;
    if (std::fseek(in.f, (long)a.offset, SEEK_SET) != 0) return MOE_ERR_INVALID_ARG;
    return std::fread(dst, 1, a.bytes, in.f) == a.bytes ? MOE_OK : MOE_ERR_INVALID_ARG;
}
