// gguf.cpp -- the GGUF model-file reader in front of the upload path.
//
// Maps a GGUF v3 file read-only and parses its header, metadata and tensor
// directory with the acceptance rules of Pixelina's loader
// (PixModelFile::open / read, src/model.cpp:138-251), so that a file the
// reference rejects is rejected here too:
//   * magic "GGUF", version 3, 1..1e6 tensors, <= 1e6 metadata pairs, all
//     header reads bounded by the first 64 MiB of the file (MODEL_MAX_HEADER);
//   * metadata values: scalar types 0..7 and 10..12, strings, arrays of
//     non-array elements (<= 1e6), booleans 0/1 only, no duplicate keys;
//   * alignment = general.alignment when present (a non-negative integer
//     value; anything else counts as invalid), else 32; a power of two
//     <= 64 MiB;
//   * tensors: rank 1..5, a type whose size weight_bytes knows (F32, F16,
//     BF16, Q8_0, Q5_K, Q6_K; src/model.cpp:87-121), offset a multiple of the
//     alignment, unique names, data inside the file after the aligned header,
//     no two tensors overlapping.
// Tensors are then uploaded through pxq_weight_upload with the Vulkan
// backend's cache identity "file:name:offset:bytes"
// (src/backend_vulkan.cpp:742-758).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <fcntl.h>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>

#include "pxq.h"

namespace pxq {
void record_error(const char* msg);
}

namespace {

constexpr uint64_t kMaxHeader = 64ull * 1024 * 1024;
constexpr uint64_t kMaxItems = 1000000;
constexpr uint32_t kMaxRank = 5;
constexpr uint64_t kDefaultAlignment = 32;
constexpr uint32_t kTypeString = 8, kTypeArray = 9, kTypeF64 = 12;

int gguf_fail(int code, const std::string& msg)
{
    pxq::record_error(msg.c_str());
    return code;
}

// Bounded little-endian cursor over the header region.
struct Cursor {
    const uint8_t* data;
    uint64_t size;  // readable bytes: min(file size, kMaxHeader)
    uint64_t pos = 0;

    bool u(unsigned bytes, uint64_t& v)
    {
        if (pos > size || bytes > size - pos) return false;
        v = 0;
        for (unsigned i = 0; i < bytes; i++) v |= (uint64_t)data[pos++] << (8 * i);
        return true;
    }
    bool str(std::string& s)
    {
        uint64_t n;
        if (!u(8, n) || n > size - pos) return false;
        s.assign(reinterpret_cast<const char*>(data + pos), (size_t)n);
        pos += n;
        return true;
    }
};

// Byte widths of the scalar value types 0..12 (0 for string / array).
constexpr unsigned kWidth[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
constexpr uint64_t kNotInteger = UINT64_MAX;

// Skip (validate) one metadata value of `type`; *as_int receives the value
// when it is a non-negative integer, else kNotInteger.
bool value(Cursor& c, uint32_t type, uint64_t* as_int)
{
    if (as_int) *as_int = kNotInteger;
    if (type == kTypeString) {
        std::string s;
        return c.str(s);
    }
    if (type == kTypeArray) {
        uint64_t elem, count;
        if (!c.u(4, elem) || !c.u(8, count) || count > kMaxItems || elem == kTypeArray) return false;
        for (uint64_t i = 0; i < count; i++)
            if (!value(c, (uint32_t)elem, nullptr)) return false;
        return true;
    }
    if (type > kTypeF64) return false;
    uint64_t raw;
    if (!c.u(kWidth[type], raw)) return false;
    if (type == 7 && raw > 1) return false;  // booleans are 0 or 1
    if (as_int) {
        switch (type) {
        case 0: case 2: case 4: case 10: *as_int = raw; break;                          // unsigned
        case 1: *as_int = (int8_t)raw < 0 ? kNotInteger : raw; break;
        case 3: *as_int = (int16_t)raw < 0 ? kNotInteger : raw; break;
        case 5: *as_int = (int32_t)raw < 0 ? kNotInteger : raw; break;
        case 11: *as_int = (int64_t)raw < 0 ? kNotInteger : raw; break;
        default: break;  // floats and booleans are not integers
        }
    }
    return true;
}

// Storage bytes of a tensor (src/model.cpp:87-121), 0 when the type or shape is not handled.
uint64_t tensor_bytes(const uint64_t* shape, uint32_t rank, uint32_t type)
{
    if (!rank || rank > kMaxRank) return 0;
    uint64_t block = 1, bytes;
    switch (type) {
    case PXQ_TYPE_F32: bytes = 4; break;
    case PXQ_TYPE_F16:
    case PXQ_TYPE_BF16: bytes = 2; break;
    case PXQ_TYPE_Q8_0: block = 32; bytes = 34; break;
    case PXQ_TYPE_Q5_K: block = 256; bytes = 176; break;
    case PXQ_TYPE_Q6_K: block = 256; bytes = 210; break;
    default: return 0;
    }
    if (!shape[0] || shape[0] % block) return 0;
    uint64_t count = shape[0] / block;
    for (uint32_t i = 1; i < rank; i++) {
        if (!shape[i] || count > UINT64_MAX / shape[i]) return 0;
        count *= shape[i];
    }
    if (count > UINT64_MAX / bytes) return 0;
    return count * bytes;
}

struct Tensor {
    std::string name;
    uint32_t type = 0, rank = 0;
    uint64_t shape[kMaxRank] = {0, 0, 0, 0, 0};
    uint64_t offset = 0, bytes = 0;
};

}  // namespace

struct pxq_gguf {
    std::string path;
    const uint8_t* data = nullptr;
    uint64_t size = 0;
    uint64_t alignment = kDefaultAlignment;
    size_t keys = 0;
    std::vector<Tensor> tensors;  // sorted by name
    ~pxq_gguf()
    {
        if (data) munmap(const_cast<uint8_t*>(data), size);
    }
};

namespace {

bool parse(pxq_gguf* f)
{
    Cursor c{f->data, std::min<uint64_t>(f->size, kMaxHeader)};
    if (f->size < 4 || std::memcmp(f->data, "GGUF", 4)) return false;
    c.pos = 4;
    uint64_t version, count, pairs;
    if (!c.u(4, version) || version != 3) return false;
    if (!c.u(8, count) || !c.u(8, pairs)) return false;
    if (!count || count > kMaxItems || pairs > kMaxItems) return false;
    std::vector<std::string> keys;
    keys.reserve((size_t)pairs);
    bool have_alignment = false;
    uint64_t alignment = kDefaultAlignment;
    for (uint64_t i = 0; i < pairs; i++) {
        std::string key;
        uint64_t type, as_int;
        if (!c.str(key) || !c.u(4, type)) return false;
        if (!value(c, (uint32_t)type, &as_int)) return false;
        if (key == "general.alignment") {
            have_alignment = true;
            alignment = as_int;
        }
        keys.push_back(std::move(key));
    }
    std::sort(keys.begin(), keys.end());
    if (std::adjacent_find(keys.begin(), keys.end()) != keys.end()) return false;  // duplicate key
    f->keys = keys.size();
    if (have_alignment && (alignment == kNotInteger)) return false;
    if (!alignment || (alignment & (alignment - 1)) || alignment > kMaxHeader) return false;
    f->alignment = alignment;
    std::vector<Tensor> ts;
    ts.reserve((size_t)count);
    for (uint64_t i = 0; i < count; i++) {
        Tensor t;
        uint64_t rank, type;
        if (!c.str(t.name) || !c.u(4, rank) || !rank || rank > kMaxRank) return false;
        t.rank = (uint32_t)rank;
        for (uint64_t d = 0; d < rank; d++)
            if (!c.u(8, t.shape[d])) return false;
        if (!c.u(4, type) || !c.u(8, t.offset)) return false;
        t.type = (uint32_t)type;
        t.bytes = tensor_bytes(t.shape, t.rank, t.type);
        if (!t.bytes || t.offset % alignment) return false;
        ts.push_back(std::move(t));
    }
    std::sort(ts.begin(), ts.end(), [](const Tensor& a, const Tensor& b) { return a.name < b.name; });
    for (size_t i = 1; i < ts.size(); i++)
        if (ts[i].name == ts[i - 1].name) return false;  // duplicate tensor name
    const uint64_t base = (c.pos + alignment - 1) & ~(alignment - 1);
    if (base > f->size) return false;
    for (Tensor& t : ts) {
        if (t.offset > f->size - base || t.bytes > f->size - base - t.offset) return false;
        t.offset += base;
    }
    // no two tensors may share bytes
    std::vector<const Tensor*> by_offset;
    for (const Tensor& t : ts) by_offset.push_back(&t);
    std::sort(by_offset.begin(), by_offset.end(), [](const Tensor* a, const Tensor* b) { return a->offset < b->offset; });
    uint64_t end = 0;
    for (const Tensor* t : by_offset) {
        if (t->offset < end) return false;
        end = t->offset + t->bytes;
    }
    f->tensors = std::move(ts);
    return !f->tensors.empty();
}

const Tensor* find(const pxq_gguf* f, const char* name)
{
    auto it = std::lower_bound(f->tensors.begin(), f->tensors.end(), name,
                               [](const Tensor& t, const char* n) { return t.name.compare(n) < 0; });
    return (it != f->tensors.end() && it->name == name) ? &*it : nullptr;
}

void fill(const Tensor& t, pxq_gguf_tensor* out)
{
    out->name = t.name.c_str();
    out->type = t.type;
    out->rank = t.rank;
    for (uint32_t d = 0; d < kMaxRank; d++) out->shape[d] = t.shape[d];
    out->offset = t.offset;
    out->bytes = t.bytes;
}

// Row geometry of a quantized 2-D (or flattened) tensor: inner = shape[0],
// rows = product of the other dimensions.
int row_view(const pxq_gguf* f, const char* name, size_t row_first, size_t row_count, const Tensor** t, size_t* first,
             size_t* count, uint64_t* row_bytes)
{
    if (!f || !name) return gguf_fail(PXQ_ERR_INVALID, "null file or name");
    *t = find(f, name);
    if (!*t) return gguf_fail(PXQ_ERR_INVALID, std::string("no tensor named ") + name);
    const Tensor& x = **t;
    if (x.type != PXQ_TYPE_Q8_0 && x.type != PXQ_TYPE_Q5_K && x.type != PXQ_TYPE_Q6_K)
        return gguf_fail(PXQ_ERR_UNSUPPORTED, std::string("tensor ") + name + " is not Q8_0, Q5_K or Q6_K");
    uint64_t rows = 1;
    for (uint32_t d = 1; d < x.rank; d++) rows *= x.shape[d];
    *row_bytes = x.bytes / rows;
    if (row_first > rows) return gguf_fail(PXQ_ERR_INVALID, "row_first beyond the tensor");
    *first = row_first;
    *count = row_count ? row_count : (size_t)(rows - row_first);
    if (!*count || *count > rows - row_first) return gguf_fail(PXQ_ERR_INVALID, "row range outside the tensor");
    return PXQ_OK;
}

}  // namespace

extern "C" {

int pxq_gguf_open(const char* path, pxq_gguf** out)
{
    if (!path || !out) return gguf_fail(PXQ_ERR_INVALID, "null path or out");
    *out = nullptr;
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return gguf_fail(PXQ_ERR_IO, std::string("cannot open ") + path);
    struct stat st;
    if (fstat(fd, &st) || !S_ISREG(st.st_mode) || st.st_size < 8) {
        ::close(fd);
        return gguf_fail(PXQ_ERR_FORMAT, std::string(path) + " is not a regular file of at least 8 bytes");
    }
    auto f = new pxq_gguf();
    f->path = path;
    f->size = (uint64_t)st.st_size;
    void* m = mmap(nullptr, (size_t)f->size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) {
        f->size = 0;
        delete f;
        return gguf_fail(PXQ_ERR_IO, std::string("cannot map ") + path);
    }
    f->data = static_cast<const uint8_t*>(m);
    if (!parse(f)) {
        delete f;
        return gguf_fail(PXQ_ERR_FORMAT, std::string(path) + " is not a GGUF v3 file this loader accepts");
    }
    *out = f;
    return PXQ_OK;
}

int pxq_gguf_close(pxq_gguf* f)
{
    delete f;
    return PXQ_OK;
}

size_t pxq_gguf_tensor_count(const pxq_gguf* f) { return f ? f->tensors.size() : 0; }

size_t pxq_gguf_metadata_count(const pxq_gguf* f) { return f ? f->keys : 0; }

const void* pxq_gguf_data(const pxq_gguf* f) { return f ? f->data : nullptr; }

int pxq_gguf_tensor_at(const pxq_gguf* f, size_t index, pxq_gguf_tensor* out)
{
    if (!f || !out) return gguf_fail(PXQ_ERR_INVALID, "null file or out");
    if (index >= f->tensors.size()) return gguf_fail(PXQ_ERR_INVALID, "tensor index out of range");
    fill(f->tensors[index], out);
    return PXQ_OK;
}

int pxq_gguf_find(const pxq_gguf* f, const char* name, pxq_gguf_tensor* out)
{
    if (!f || !name || !out) return gguf_fail(PXQ_ERR_INVALID, "null file, name or out");
    const Tensor* t = find(f, name);
    if (!t) return gguf_fail(PXQ_ERR_INVALID, std::string("no tensor named ") + name);
    fill(*t, out);
    return PXQ_OK;
}

int pxq_gguf_upload(pxq_gguf* f, const char* name, size_t row_first, size_t row_count, pxq_weight** out)
{
    if (!out) return gguf_fail(PXQ_ERR_INVALID, "null out");
    const Tensor* t;
    size_t first, count;
    uint64_t row_bytes;
    if (int rc = row_view(f, name, row_first, row_count, &t, &first, &count, &row_bytes)) return rc;
    const uint64_t offset = t->offset + first * row_bytes, bytes = count * row_bytes;
    const std::string key = f->path + ":" + t->name + ":" + std::to_string(offset) + ":" + std::to_string(bytes);
    return pxq_weight_upload(f->data + offset, 0, t->type, (size_t)t->shape[0], count, key.c_str(), out);
}

int pxq_gguf_upload_gated(pxq_gguf* f, const char* gate, size_t gate_first, const char* up, size_t up_first, size_t rows,
                          pxq_weight** out)
{
    if (!out || !rows) return gguf_fail(PXQ_ERR_INVALID, "null out or zero rows");
    const Tensor *tg, *tu;
    size_t fg, fu, cg, cu;
    uint64_t bg, bu;
    if (int rc = row_view(f, gate, gate_first, rows, &tg, &fg, &cg, &bg)) return rc;
    if (int rc = row_view(f, up, up_first, rows, &tu, &fu, &cu, &bu)) return rc;
    if (tg->type != tu->type || tg->shape[0] != tu->shape[0])
        return gguf_fail(PXQ_ERR_INVALID, "gate and up differ in type or inner size");
    const uint64_t og = tg->offset + fg * bg, ou = tu->offset + fu * bu;
    const std::string key = f->path + ":" + tg->name + ":" + std::to_string(og) + "+" + tu->name + ":" + std::to_string(ou) +
                            ":" + std::to_string(rows * bg) + ":gated";
    return pxq_weight_upload_gated(f->data + og, f->data + ou, 0, tg->type, (size_t)tg->shape[0], rows, key.c_str(), out);
}

}  // extern "C"
