// .tmod weight files -> device memory (vox_cuda_tmod_*): the on-disk step before the Q8/Q4 operators.
//
// Vox's own container (src/formats.hpp:44-90, reader src/formats.cpp:175-205, writer :215-249): a 64-byte header
// ("VOXM", version 1.x, flags, manifest and data ranges), a JSON manifest whose "blobs" object maps each tensor name
// to {dtype, shape, offset, nbytes}, and a data area of blobs aligned to 4096 bytes for mmap. Vox maps the file and,
// with a GPU, copies every weight into video memory (upload_parts, gpu_vulkan.cpp:476-536), Q8/Q4 matrices as codes
// plus a "<name>.scale" f32 blob (nn::mat_named, nn.cpp:132-145).
//
// Here the file is mapped read-only and, on the first upload, page-locked for the device (read-only host
// registration): each blob is then one cudaMemcpyAsync straight from the mapping, no host copy. Where registration is
// not available a ring of pinned staging buffers owned by the handle is used instead: host threads copy chunk i of
// the mapping into a free staging buffer while the copy engine moves chunk i-1 to the device, so page-cache reads,
// host copies and PCIe transfers overlap. Q8/Q4 matrices can be dequantised on arrival (vox_cuda_tmod_upload_dequant), bit-exact with
// mat_row. The manifest is read by a small JSON reader that accepts the whole JSON grammar (the manifest carries model
// configuration besides the blob table) and keeps only the blob table.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"

struct vox_cuda_tmod {
    struct Blob {
        int dtype = 0;
        std::vector<int64_t> shape;
        uint64_t offset = 0, nbytes = 0;  // offset from the start of the file
    };
    std::string path;
    const uint8_t *map = nullptr;
    size_t size = 0;
    uint32_t flags = 0;
    std::vector<std::string> names;  // manifest order
    std::map<std::string, Blob> blobs;
    // pinned staging ring (allocated on the first upload) and the events that free its buffers
    std::mutex mu;
    std::vector<void *> stage;
    std::vector<cudaEvent_t> done;
    int device = -1;
    bool registered = false;  // the mapping is page-locked for the device: blobs are copied from it directly
};

namespace voxcuda {
namespace {

constexpr size_t kStageBytes = size_t(32) << 20;  // one staging buffer
constexpr int kStages = 4;
constexpr int kCopyThreads = 8;                    // host threads per staging copy

// ------------------------------------------------------------------ JSON (RFC 8259) reader, values kept as needed
struct Json {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    std::string s;      // Str
    double num = 0;     // Num (also kept as text for exact integers)
    std::string text;   // Num: the literal
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
    const Json *get(const std::string &k) const {
        for (auto &kv : obj)
            if (kv.first == k) return &kv.second;
        return nullptr;
    }
};

struct JsonReader {
    const char *p, *e;
    std::string err;
    int depth = 0;
    void ws() {
        while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
    }
    bool fail(const char *m) {
        if (err.empty()) err = m;
        return false;
    }
    static void put_utf8(std::string &o, uint32_t c) {
        if (c < 0x80) o += char(c);
        else if (c < 0x800) o += char(0xC0 | (c >> 6)), o += char(0x80 | (c & 0x3F));
        else if (c < 0x10000) o += char(0xE0 | (c >> 12)), o += char(0x80 | ((c >> 6) & 0x3F)), o += char(0x80 | (c & 0x3F));
        else o += char(0xF0 | (c >> 18)), o += char(0x80 | ((c >> 12) & 0x3F)), o += char(0x80 | ((c >> 6) & 0x3F)), o += char(0x80 | (c & 0x3F));
    }
    bool hex4(uint32_t &v) {
        if (e - p < 4) return fail("short \\u escape");
        v = 0;
        for (int i = 0; i < 4; ++i, ++p) {
            const char c = *p;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= uint32_t(c - '0');
            else if (c >= 'a' && c <= 'f') v |= uint32_t(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= uint32_t(c - 'A' + 10);
            else return fail("bad \\u escape");
        }
        return true;
    }
    bool str(std::string &o) {
        if (p >= e || *p != '"') return fail("string expected");
        ++p;
        while (p < e && *p != '"') {
            const unsigned char c = static_cast<unsigned char>(*p);
            if (c < 0x20) return fail("control character in string");
            if (c != '\\') {
                o += char(c);
                ++p;
                continue;
            }
            if (++p >= e) return fail("bad escape");
            const char x = *p++;
            switch (x) {
                case '"': o += '"'; break;
                case '\\': o += '\\'; break;
                case '/': o += '/'; break;
                case 'b': o += '\b'; break;
                case 'f': o += '\f'; break;
                case 'n': o += '\n'; break;
                case 'r': o += '\r'; break;
                case 't': o += '\t'; break;
                case 'u': {
                    uint32_t v;
                    if (!hex4(v)) return false;
                    if (v >= 0xD800 && v < 0xDC00) {  // surrogate pair
                        uint32_t lo;
                        if (e - p < 2 || p[0] != '\\' || p[1] != 'u') return fail("lone surrogate");
                        p += 2;
                        if (!hex4(lo) || lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair");
                        v = 0x10000 + ((v - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    put_utf8(o, v);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p >= e) return fail("unterminated string");
        ++p;
        return true;
    }
    bool value(Json &v) {
        if (++depth > 512) return fail("nesting too deep");
        ws();
        if (p >= e) return fail("value expected");
        bool ok = true;
        if (*p == '{') {
            v.kind = Json::Obj;
            ++p;
            ws();
            if (p < e && *p == '}') ++p;
            else
                for (;;) {
                    std::string k;
                    ws();
                    if (!str(k)) return false;
                    ws();
                    if (p >= e || *p != ':') return fail("':' expected");
                    ++p;
                    v.obj.emplace_back(std::move(k), Json());
                    if (!value(v.obj.back().second)) return false;
                    ws();
                    if (p < e && *p == ',') { ++p; continue; }
                    if (p < e && *p == '}') { ++p; break; }
                    return fail("',' or '}' expected");
                }
        } else if (*p == '[') {
            v.kind = Json::Arr;
            ++p;
            ws();
            if (p < e && *p == ']') ++p;
            else
                for (;;) {
                    v.arr.emplace_back();
                    if (!value(v.arr.back())) return false;
                    ws();
                    if (p < e && *p == ',') { ++p; continue; }
                    if (p < e && *p == ']') { ++p; break; }
                    return fail("',' or ']' expected");
                }
        } else if (*p == '"') {
            v.kind = Json::Str;
            ok = str(v.s);
        } else if (e - p >= 4 && !std::strncmp(p, "true", 4)) {
            v.kind = Json::Bool, v.num = 1, p += 4;
        } else if (e - p >= 5 && !std::strncmp(p, "false", 5)) {
            v.kind = Json::Bool, v.num = 0, p += 5;
        } else if (e - p >= 4 && !std::strncmp(p, "null", 4)) {
            v.kind = Json::Null, p += 4;
        } else {
            const char *b = p;
            if (p < e && *p == '-') ++p;
            if (p >= e || !(*p >= '0' && *p <= '9')) return fail("bad number");
            if (*p == '0') ++p;
            else
                while (p < e && *p >= '0' && *p <= '9') ++p;
            if (p < e && *p == '.') {
                ++p;
                if (p >= e || !(*p >= '0' && *p <= '9')) return fail("bad number");
                while (p < e && *p >= '0' && *p <= '9') ++p;
            }
            if (p < e && (*p == 'e' || *p == 'E')) {
                ++p;
                if (p < e && (*p == '+' || *p == '-')) ++p;
                if (p >= e || !(*p >= '0' && *p <= '9')) return fail("bad number");
                while (p < e && *p >= '0' && *p <= '9') ++p;
            }
            v.kind = Json::Num;
            v.text.assign(b, size_t(p - b));
            v.num = std::strtod(v.text.c_str(), nullptr);
        }
        --depth;
        return ok;
    }
};

// a non-negative integer JSON number, exactly (offsets and sizes exceed 2^53 only in files we would reject anyway)
bool as_u64(const Json *j, uint64_t &out) {
    if (!j || j->kind != Json::Num || j->text.empty() || j->text[0] == '-') return false;
    for (char c : j->text)
        if (c < '0' || c > '9') return false;
    if (j->text.size() > 19) return false;
    out = std::strtoull(j->text.c_str(), nullptr, 10);
    return true;
}

// Vox's DType order (src/common.hpp:22) and names (src/formats.cpp:34-55)
const char *const kDtypeNames[] = {"F32", "F16", "BF16", "I32", "I16", "I8", "U8"};

int tmod_error(int status, const std::string &m) { return set_error(status, m); }

#pragma pack(push, 1)
struct TmodHeader {
    char magic[4];
    uint16_t version_major, version_minor;
    uint32_t flags, reserved0;
    uint64_t manifest_offset, manifest_size, data_offset, data_size;
    uint8_t reserved[16];
};
#pragma pack(pop)
static_assert(sizeof(TmodHeader) == 64, "the .tmod header is 64 bytes");

int parse(vox_cuda_tmod &t) {
    const std::string &path = t.path;
    if (t.size < sizeof(TmodHeader)) return tmod_error(VOX_CUDA_ERR_FORMAT, "file too small for .tmod: " + path);
    TmodHeader h;
    std::memcpy(&h, t.map, sizeof h);
    if (std::memcmp(h.magic, "VOXM", 4) != 0) return tmod_error(VOX_CUDA_ERR_FORMAT, "not a .tmod file: " + path);
    if (h.version_major != 1)
        return tmod_error(VOX_CUDA_ERR_FORMAT, ".tmod format " + std::to_string(h.version_major) + ".x is not supported");
    if (h.manifest_offset > t.size || h.manifest_size > t.size - h.manifest_offset || h.data_offset > t.size ||
        h.data_size > t.size - h.data_offset)
        return tmod_error(VOX_CUDA_ERR_FORMAT, "truncated .tmod: " + path);
    t.flags = h.flags;
    JsonReader r{reinterpret_cast<const char *>(t.map + h.manifest_offset),
                 reinterpret_cast<const char *>(t.map + h.manifest_offset + h.manifest_size), {}};
    Json m;
    if (!r.value(m)) return tmod_error(VOX_CUDA_ERR_FORMAT, "bad .tmod manifest: " + r.err);
    r.ws();
    if (r.p != r.e) return tmod_error(VOX_CUDA_ERR_FORMAT, "bad .tmod manifest: trailing characters");
    if (m.kind != Json::Obj) return tmod_error(VOX_CUDA_ERR_FORMAT, "bad .tmod manifest: not an object");
    const Json *blobs = m.get("blobs");
    if (!blobs) return VOX_CUDA_OK;  // a file without tensors
    if (blobs->kind != Json::Obj) return tmod_error(VOX_CUDA_ERR_FORMAT, "bad .tmod manifest: blobs is not an object");
    for (auto &kv : blobs->obj) {
        const Json &b = kv.second;
        vox_cuda_tmod::Blob bl;
        const Json *dt = b.get("dtype"), *sh = b.get("shape");
        if (!dt || dt->kind != Json::Str || !sh || sh->kind != Json::Arr)
            return tmod_error(VOX_CUDA_ERR_FORMAT, "bad blob entry: " + kv.first);
        bl.dtype = -1;
        for (int i = 0; i < 7; ++i)
            if (dt->s == kDtypeNames[i]) bl.dtype = i;
        if (bl.dtype < 0) return tmod_error(VOX_CUDA_ERR_FORMAT, "unsupported dtype: " + dt->s);
        for (auto &d : sh->arr) {
            uint64_t v;
            if (!as_u64(&d, v) || v > (uint64_t(1) << 62)) return tmod_error(VOX_CUDA_ERR_FORMAT, "bad shape: " + kv.first);
            bl.shape.push_back(int64_t(v));
        }
        uint64_t off, n;
        if (!as_u64(b.get("offset"), off) || !as_u64(b.get("nbytes"), n))
            return tmod_error(VOX_CUDA_ERR_FORMAT, "bad blob entry: " + kv.first);
        if (off > h.data_size || n > h.data_size - off) return tmod_error(VOX_CUDA_ERR_FORMAT, "blob out of range: " + kv.first);
        bl.offset = h.data_offset + off;
        bl.nbytes = n;
        if (!t.blobs.count(kv.first)) t.names.push_back(kv.first);
        t.blobs[kv.first] = std::move(bl);
    }
    return VOX_CUDA_OK;
}

// The handle's transfer path on the current device, set up on first use: the mapping itself page-locked for the
// device (read-only registration; copies then go straight from the page cache, no host copy), or, where that is not
// supported or VOX_CUDA_TMOD_REGISTER=0, the pinned staging ring.
int ensure_stage(vox_cuda_tmod &t) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch("vox_cuda_tmod_upload");
    if ((!t.stage.empty() || t.registered) && t.device == dev) return VOX_CUDA_OK;
    if (!t.stage.empty() || t.registered)
        return set_error(VOX_CUDA_ERR_ARG, "vox_cuda_tmod_upload: the handle's first upload used another device");
    const char *env = std::getenv("VOX_CUDA_TMOD_REGISTER");
    int ro = 0;
    if (t.size > 0 && !(env && env[0] == '0') && cudaDeviceGetAttribute(&ro, cudaDevAttrHostRegisterReadOnlySupported, dev) == cudaSuccess &&
        ro) {
        if (cudaHostRegister(const_cast<uint8_t *>(t.map), t.size, cudaHostRegisterReadOnly) == cudaSuccess) {
            t.registered = true;
            t.device = dev;
            return VOX_CUDA_OK;
        }
        cudaGetLastError();  // not available for this mapping: use the staging ring
    }
    for (int i = 0; i < kStages; ++i) {
        void *p = nullptr;
        cudaEvent_t ev;
        if (cudaHostAlloc(&p, kStageBytes, cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            return set_error(VOX_CUDA_ERR_OOM, "vox_cuda_tmod_upload: cannot allocate pinned staging memory");
        }
        if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
            cudaFreeHost(p);
            return check_launch("vox_cuda_tmod_upload");
        }
        t.stage.push_back(p);
        t.done.push_back(ev);
    }
    t.device = dev;
    return VOX_CUDA_OK;
}

// host copy of n bytes split over up to kCopyThreads threads (large chunks only)
void par_copy(void *dst, const void *src, size_t n) {
    if (n < (size_t(2) << 20)) {
        std::memcpy(dst, src, n);
        return;
    }
    const size_t part = (n / kCopyThreads + 4095) / 4096 * 4096;
    std::thread th[kCopyThreads - 1];
    int used = 0;
    for (int i = 1; i < kCopyThreads && size_t(i) * part < n; ++i, ++used) {
        const size_t o = size_t(i) * part, len = n - o < part ? n - o : part;
        th[i - 1] = std::thread([=] { std::memcpy(static_cast<char *>(dst) + o, static_cast<const char *>(src) + o, len); });
    }
    std::memcpy(dst, src, n < part ? n : part);
    for (int i = 0; i < used; ++i) th[i].join();
}

// bytes [src, src + n) of the mapping -> device dst, through the ring, on stream st
int staged_copy(vox_cuda_tmod &t, void *dst, const uint8_t *src, uint64_t n, cudaStream_t st, int &slot) {
    for (uint64_t o = 0; o < n; o += kStageBytes) {
        const size_t len = size_t(n - o < kStageBytes ? n - o : kStageBytes);
        // the buffer's previous transfer must have left it (its event: recorded after that copy)
        if (cudaEventSynchronize(t.done[slot]) != cudaSuccess) return check_launch("vox_cuda_tmod_upload");
        par_copy(t.stage[slot], src + o, len);
        if (cudaMemcpyAsync(static_cast<uint8_t *>(dst) + o, t.stage[slot], len, cudaMemcpyHostToDevice, st) != cudaSuccess ||
            cudaEventRecord(t.done[slot], st) != cudaSuccess)
            return check_launch("vox_cuda_tmod_upload");
        slot = (slot + 1) % kStages;
    }
    return VOX_CUDA_OK;
}

const vox_cuda_tmod::Blob *find(const vox_cuda_tmod *t, const char *name) {
    if (!t || !name) return nullptr;
    auto it = t->blobs.find(name);
    return it == t->blobs.end() ? nullptr : &it->second;
}

}  // namespace
}  // namespace voxcuda

using namespace voxcuda;

extern "C" {

int vox_cuda_tmod_open(const char *path, vox_cuda_tmod **out) {
    VOX_REQUIRE(path && out, "vox_cuda_tmod_open: NULL argument");
    *out = nullptr;
    auto t = std::make_unique<vox_cuda_tmod>();
    t->path = path;
    const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return set_error(VOX_CUDA_ERR_IO, std::string("cannot open ") + path);
    struct stat stt;
    if (fstat(fd, &stt) != 0) {
        ::close(fd);
        return set_error(VOX_CUDA_ERR_IO, std::string("cannot stat ") + path);
    }
    t->size = size_t(stt.st_size);
    if (t->size > 0) {
        void *p = mmap(nullptr, t->size, PROT_READ, MAP_PRIVATE, fd, 0);
        if (p == MAP_FAILED) {
            ::close(fd);
            return set_error(VOX_CUDA_ERR_IO, std::string("cannot map ") + path);
        }
        t->map = static_cast<const uint8_t *>(p);
    }
    ::close(fd);
    const int rc = parse(*t);
    if (rc != VOX_CUDA_OK) {
        vox_cuda_tmod_close(t.release());
        return rc;
    }
    *out = t.release();
    return VOX_CUDA_OK;
}

void vox_cuda_tmod_close(vox_cuda_tmod *t) {
    if (!t) return;
    if (t->registered) {  // copies from the mapping may still be in flight on the caller's streams
        cudaDeviceSynchronize();
        cudaHostUnregister(const_cast<uint8_t *>(t->map));
    }
    for (auto ev : t->done) {
        cudaEventSynchronize(ev);
        cudaEventDestroy(ev);
    }
    for (void *p : t->stage) cudaFreeHost(p);
    if (t->map) munmap(const_cast<uint8_t *>(t->map), t->size);
    delete t;
}

int vox_cuda_tmod_count(const vox_cuda_tmod *t, int64_t *n) {
    VOX_REQUIRE(t && n, "vox_cuda_tmod_count: NULL argument");
    *n = int64_t(t->names.size());
    return VOX_CUDA_OK;
}

int vox_cuda_tmod_name(const vox_cuda_tmod *t, int64_t i, const char **name) {
    VOX_REQUIRE(t && name, "vox_cuda_tmod_name: NULL argument");
    VOX_REQUIRE(i >= 0 && i < int64_t(t->names.size()), "vox_cuda_tmod_name: index out of range");
    *name = t->names[size_t(i)].c_str();
    return VOX_CUDA_OK;
}

int vox_cuda_tmod_info(const vox_cuda_tmod *t, const char *name, int *dtype, int64_t *shape, int *ndim, uint64_t *nbytes) {
    VOX_REQUIRE(t && name, "vox_cuda_tmod_info: NULL argument");
    const auto *b = find(t, name);
    if (!b) return set_error(VOX_CUDA_ERR_FORMAT, std::string("missing blob in .tmod: ") + name);
    if (dtype) *dtype = b->dtype;
    if (ndim) *ndim = int(b->shape.size());
    if (shape)
        for (size_t i = 0; i < b->shape.size() && i < VOX_CUDA_TMOD_MAX_DIMS; ++i) shape[i] = b->shape[i];
    if (nbytes) *nbytes = b->nbytes;
    return VOX_CUDA_OK;
}

int vox_cuda_tmod_data(const vox_cuda_tmod *t, const char *name, const void **host) {
    VOX_REQUIRE(t && name && host, "vox_cuda_tmod_data: NULL argument");
    const auto *b = find(t, name);
    if (!b) return set_error(VOX_CUDA_ERR_FORMAT, std::string("missing blob in .tmod: ") + name);
    *host = t->map + b->offset;
    return VOX_CUDA_OK;
}

int vox_cuda_tmod_upload(vox_cuda_tmod *t, const char *const *names, int64_t count, void *const *dst, void *stream) {
    VOX_REQUIRE(t && count >= 0 && (count == 0 || (names && dst)), "vox_cuda_tmod_upload: bad arguments");
    std::lock_guard<std::mutex> lk(t->mu);
    int rc = ensure_stage(*t);
    if (rc != VOX_CUDA_OK) return rc;
    int slot = 0;
    for (int64_t i = 0; i < count; ++i) {
        const auto *b = find(t, names[i]);
        if (!b) return set_error(VOX_CUDA_ERR_FORMAT, std::string("missing blob in .tmod: ") + (names[i] ? names[i] : "(null)"));
        VOX_REQUIRE(dst[i] != nullptr || b->nbytes == 0, "vox_cuda_tmod_upload: NULL destination");
        if (t->registered) {
            if (b->nbytes && cudaMemcpyAsync(dst[i], t->map + b->offset, b->nbytes, cudaMemcpyHostToDevice,
                                             reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess)
                return check_launch("vox_cuda_tmod_upload");
            continue;
        }
        rc = staged_copy(*t, dst[i], t->map + b->offset, b->nbytes, reinterpret_cast<cudaStream_t>(stream), slot);
        if (rc != VOX_CUDA_OK) return rc;
    }
    return VOX_CUDA_OK;
}

int vox_cuda_tmod_upload_dequant(vox_cuda_tmod *t, const char *name, void *dst, int out_dtype, void *stream) {
    VOX_REQUIRE(t && name && dst, "vox_cuda_tmod_upload_dequant: NULL argument");
    VOX_REQUIRE(out_dtype == VOX_CUDA_F32 || out_dtype == VOX_CUDA_BF16, "vox_cuda_tmod_upload_dequant: out dtype must be F32 or BF16");
    const auto *b = find(t, name);
    const auto *s = find(t, (std::string(name) + ".scale").c_str());
    if (!b) return set_error(VOX_CUDA_ERR_FORMAT, std::string("missing blob in .tmod: ") + name);
    if (!s) return set_error(VOX_CUDA_ERR_FORMAT, std::string("missing blob in .tmod: ") + name + ".scale");
    // nn::mat_named (nn.cpp:132-145): I8 -> Q8, U8 -> Q4 (cols = 2 x the stored width), scales F32 [rows][cols/32]
    if (b->dtype != 5 && b->dtype != 6) return set_error(VOX_CUDA_ERR_FORMAT, std::string("not a Q8/Q4 matrix: ") + name);
    if (s->dtype != 0) return set_error(VOX_CUDA_ERR_FORMAT, std::string("quantization scales must be F32: ") + name);
    const bool q4 = b->dtype == 6;
    const int64_t rows = b->shape.empty() ? 0 : b->shape[0];
    const int64_t cols = (b->shape.size() > 1 ? b->shape[1] : 1) * (q4 ? 2 : 1);
    if (rows <= 0 || cols % 32 != 0 || b->nbytes != uint64_t(rows) * uint64_t(q4 ? cols / 2 : cols) ||
        s->nbytes != uint64_t(rows) * uint64_t(cols / 32) * 4)
        return set_error(VOX_CUDA_ERR_FORMAT, std::string("inconsistent Q8/Q4 blob sizes: ") + name);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    void *codes = nullptr, *scales = nullptr;
    if (cudaMallocAsync(&codes, b->nbytes, st) != cudaSuccess || cudaMallocAsync(&scales, s->nbytes, st) != cudaSuccess) {
        cudaGetLastError();
        if (codes) cudaFreeAsync(codes, st);
        return set_error(VOX_CUDA_ERR_OOM, "vox_cuda_tmod_upload_dequant: cannot allocate device staging");
    }
    const char *nm[2] = {name, nullptr};
    const std::string sname = std::string(name) + ".scale";
    nm[1] = sname.c_str();
    void *d[2] = {codes, scales};
    int rc = vox_cuda_tmod_upload(t, nm, 2, d, stream);
    if (rc == VOX_CUDA_OK)
        rc = q4 ? vox_cuda_dequant_q4(static_cast<const uint8_t *>(codes), scales, VOX_CUDA_F32, dst, out_dtype, rows, cols, stream)
                : vox_cuda_dequant_q8(static_cast<const int8_t *>(codes), scales, VOX_CUDA_F32, dst, out_dtype, rows, cols, stream);
    cudaFreeAsync(codes, st);
    cudaFreeAsync(scales, st);
    return rc;
}

}  // extern "C"
