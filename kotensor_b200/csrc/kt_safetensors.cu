// kt_safetensors.cu -- the reference's safetensors model files between disk and HBM.
//
// Format (Engine/kotensor/src/main/kotlin/SafeTensors.kt): an 8-byte
// little-endian header length L, L bytes of UTF-8 JSON, then the tensors' bytes.
// The JSON is an object; every member whose value is an object is a tensor
// {"dtype", "shape", "data_offsets": [start, end)} with offsets counted from the
// end of the header, except "__metadata__", a string map.  The writer
// (SafeTensors.saveEntries, SafeTensors.kt:220-249) puts "__metadata__" first
// when it is not empty, then the tensors in the caller's order with no gaps
// between their bytes, and pads the header with spaces to a multiple of 8.
//
// Host side: the header is parsed here (a small JSON reader with the
// reference's number and escape rules, JsonParser.kt:3-162) and tensor bytes
// are read with pread, so several threads may read one file.  Device side:
// each file owns two pinned staging buffers of kChunk bytes; chunk i+1 is read
// from the file while chunk i is copied to HBM, and an event per buffer keeps a
// buffer from being refilled before its copy (and, for converting reads, the
// conversion kernel that reads its device twin) has finished.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <unordered_map>

#include "kt_internal.h"

namespace {

constexpr size_t kChunk = static_cast<size_t>(16) << 20;       // bytes per staging buffer
constexpr int64_t kMaxHeader = static_cast<int64_t>(100) << 20;  // SafeTensors.kt:42
constexpr int kMaxRank = 8;
constexpr int kMaxDepth = 128;  // JSON nesting accepted by the header reader

// A failed check (-> KT_ERR_INVALID_ARGUMENT, the reference's require) or a
// failed system call (-> KT_ERR_IO, the reference's IOException).
struct StError : std::runtime_error {
    kt_status status;
    StError(kt_status s, const std::string& m) : std::runtime_error(m), status(s) {}
};
[[noreturn]] void bad(const std::string& m) { throw StError(KT_ERR_INVALID_ARGUMENT, m); }
[[noreturn]] void io_error(const std::string& m) { throw StError(KT_ERR_IO, m + ": " + std::strerror(errno)); }
[[noreturn]] void cuda_error(cudaError_t e, const std::string& m) {
    throw StError(e == cudaErrorMemoryAllocation ? KT_ERR_OUT_OF_MEMORY : KT_ERR_CUDA,
                  m + ": " + cudaGetErrorString(e));
}
void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) cuda_error(e, what);
}

// ------------------------------------------------------------------ JSON
struct JValue {
    enum Kind { Null, Bool, Int, Real, Str, Arr, Obj } kind = Null;
    bool b = false;
    int64_t i = 0;
    double d = 0.0;
    std::string s;  // a string's value, or a number's literal text
    std::vector<JValue> arr;
    std::vector<std::pair<std::string, JValue>> obj;
};

void append_utf8(std::string& out, uint32_t cp) {
    if (cp < 0x80) {
        out.push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
        out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else if (cp < 0x10000) {
        out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
        out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
        out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
        out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
        out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
        out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
}

// Recursive-descent reader with the reference's rules: whitespace is space,
// \n, \r, \t; a number is -?digits(.digits)?([eE][+-]?digits)? and is an
// integer when it has neither fraction nor exponent and fits 64 bits; a
// repeated key keeps its first position and its last value (LinkedHashMap).
class JsonReader {
public:
    JsonReader(const char* p, size_t n) : begin_(p), p_(p), end_(p + n) {}

    JValue document() {
        skip_ws();
        JValue v = value(0);
        skip_ws();
        if (p_ != end_) bad("Unexpected trailing content at " + pos());
        return v;
    }

private:
    const char* begin_;
    const char* p_;
    const char* end_;

    std::string pos() const { return std::to_string(p_ - begin_); }
    char peek() const {
        if (p_ >= end_) bad("Unexpected end of JSON");
        return *p_;
    }
    void skip_ws() {
        while (p_ < end_ && (*p_ == ' ' || *p_ == '\n' || *p_ == '\r' || *p_ == '\t')) ++p_;
    }

    JValue value(int depth) {
        if (depth > kMaxDepth) bad("JSON nested deeper than " + std::to_string(kMaxDepth));
        const char c = peek();
        if (c == '{') return object(depth);
        if (c == '[') return array(depth);
        if (c == '"') {
            JValue v;
            v.kind = JValue::Str;
            v.s = string();
            return v;
        }
        if (c == 't') return literal("true", JValue::Bool, true);
        if (c == 'f') return literal("false", JValue::Bool, false);
        if (c == 'n') return literal("null", JValue::Null, false);
        if (c == '-' || (c >= '0' && c <= '9')) return number();
        bad(std::string("Unexpected character '") + c + "' at " + pos());
    }

    JValue literal(const char* word, JValue::Kind kind, bool b) {
        const size_t n = std::strlen(word);
        if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, word, n) != 0) bad("Unexpected literal at " + pos());
        p_ += n;
        JValue v;
        v.kind = kind;
        v.b = b;
        return v;
    }

    JValue object(int depth) {
        ++p_;
        JValue v;
        v.kind = JValue::Obj;
        skip_ws();
        if (peek() == '}') {
            ++p_;
            return v;
        }
        while (true) {
            skip_ws();
            if (peek() != '"') bad("Expected a string key at " + pos());
            std::string key = string();
            skip_ws();
            if (peek() != ':') bad("Expected ':' at " + pos());
            ++p_;
            skip_ws();
            JValue member = value(depth + 1);
            bool replaced = false;
            for (auto& kv : v.obj)
                if (kv.first == key) {
                    kv.second = std::move(member);
                    replaced = true;
                    break;
                }
            if (!replaced) v.obj.emplace_back(std::move(key), std::move(member));
            skip_ws();
            const char c = peek();
            if (c == ',') {
                ++p_;
            } else if (c == '}') {
                ++p_;
                return v;
            } else {
                bad("Expected ',' or '}' at " + pos());
            }
        }
    }

    JValue array(int depth) {
        ++p_;
        JValue v;
        v.kind = JValue::Arr;
        skip_ws();
        if (peek() == ']') {
            ++p_;
            return v;
        }
        while (true) {
            skip_ws();
            v.arr.push_back(value(depth + 1));
            skip_ws();
            const char c = peek();
            if (c == ',') {
                ++p_;
            } else if (c == ']') {
                ++p_;
                return v;
            } else {
                bad("Expected ',' or ']' at " + pos());
            }
        }
    }

    uint32_t hex4() {
        if (end_ - p_ < 4) bad("Truncated \\u escape");
        uint32_t v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = *p_++;
            v <<= 4;
            if (c >= '0' && c <= '9') v |= static_cast<uint32_t>(c - '0');
            else if (c >= 'a' && c <= 'f') v |= static_cast<uint32_t>(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= static_cast<uint32_t>(c - 'A' + 10);
            else bad("Invalid \\u escape at " + pos());
        }
        return v;
    }

    std::string string() {
        ++p_;
        std::string out;
        while (true) {
            if (p_ >= end_) bad("Unterminated string");
            const char c = *p_++;
            if (c == '"') return out;
            if (c != '\\') {
                out.push_back(c);
                continue;
            }
            if (p_ >= end_) bad("Unterminated escape");
            const char e = *p_++;
            switch (e) {
                case '"': out.push_back('"'); break;
                case '\\': out.push_back('\\'); break;
                case '/': out.push_back('/'); break;
                case 'b': out.push_back('\b'); break;
                case 'f': out.push_back('\f'); break;
                case 'n': out.push_back('\n'); break;
                case 'r': out.push_back('\r'); break;
                case 't': out.push_back('\t'); break;
                case 'u': {
                    uint32_t cp = hex4();
                    // A UTF-16 surrogate pair written as two escapes is one code point.
                    if (cp >= 0xD800 && cp < 0xDC00 && end_ - p_ >= 6 && p_[0] == '\\' && p_[1] == 'u') {
                        const char* save = p_;
                        p_ += 2;
                        const uint32_t lo = hex4();
                        if (lo >= 0xDC00 && lo < 0xE000) cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                        else p_ = save;
                    }
                    append_utf8(out, cp);
                    break;
                }
                default:
                    bad(std::string("Invalid escape '\\") + e + "' at " + std::to_string(p_ - begin_ - 1));
            }
        }
    }

    JValue number() {
        const char* start = p_;
        bool integral = true;
        if (*p_ == '-') ++p_;
        while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        if (p_ < end_ && *p_ == '.') {
            integral = false;
            ++p_;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        if (p_ < end_ && (*p_ == 'e' || *p_ == 'E')) {
            integral = false;
            ++p_;
            if (p_ < end_ && (*p_ == '+' || *p_ == '-')) ++p_;
            while (p_ < end_ && *p_ >= '0' && *p_ <= '9') ++p_;
        }
        JValue v;
        v.s.assign(start, p_);
        if (integral) {
            errno = 0;
            char* stop = nullptr;
            const long long x = std::strtoll(v.s.c_str(), &stop, 10);
            if (errno == 0 && stop && *stop == '\0' && !v.s.empty() && v.s != "-") {
                v.kind = JValue::Int;
                v.i = x;
                return v;
            }
        }
        char* stop = nullptr;
        const double x = std::strtod(v.s.c_str(), &stop);
        if (!stop || *stop != '\0' || v.s.empty() || v.s == "-") bad("Invalid number '" + v.s + "'");
        v.kind = JValue::Real;
        v.d = x;
        return v;
    }
};

// Number.toLong() / toInt() of a parsed number (a fraction is truncated).
int64_t as_long(const JValue& v, const std::string& what) {
    if (v.kind == JValue::Int) return v.i;
    if (v.kind == JValue::Real) return static_cast<int64_t>(v.d);
    bad(what + " is not a number");
}

// Metadata values are strings in files the reference writes; other JSON
// values keep their text (numbers as written, true / false / null).
std::string as_text(const JValue& v) {
    switch (v.kind) {
        case JValue::Str:
        case JValue::Int:
        case JValue::Real: return v.s;
        case JValue::Bool: return v.b ? "true" : "false";
        case JValue::Null: return "null";
        default: return v.kind == JValue::Arr ? "[...]" : "{...}";
    }
}

// ------------------------------------------------------------------ files
void pread_full(int fd, void* dst, size_t n, int64_t offset) {
    auto* p = static_cast<uint8_t*>(dst);
    while (n > 0) {
        const ssize_t r = ::pread(fd, p, n, static_cast<off_t>(offset));
        if (r < 0) {
            if (errno == EINTR) continue;
            io_error("read failed");
        }
        if (r == 0) {
            errno = EIO;
            io_error("unexpected end of file");
        }
        p += r;
        n -= static_cast<size_t>(r);
        offset += r;
    }
}

// Large reads in parallel slices: one thread moves a few GB/s out of the page
// cache, less than a pinned host-to-device copy takes.
void read_parallel(int fd, void* dst, size_t n, int64_t offset) {
    constexpr size_t kSlice = static_cast<size_t>(4) << 20;
    const size_t parts = std::min<size_t>(4, (n + kSlice - 1) / kSlice);
    if (parts <= 1) {
        pread_full(fd, dst, n, offset);
        return;
    }
    std::vector<std::thread> threads;
    std::vector<std::string> errors(parts);
    std::vector<int> codes(parts, 0);
    const size_t per = (n + parts - 1) / parts;
    for (size_t t = 0; t < parts; ++t) {
        const size_t b = t * per, e = std::min(n, b + per);
        threads.emplace_back([&, t, b, e] {
            try {
                pread_full(fd, static_cast<uint8_t*>(dst) + b, e - b, offset + static_cast<int64_t>(b));
            } catch (const StError& err) {
                errors[t] = err.what();
                codes[t] = err.status;
            }
        });
    }
    for (auto& th : threads) th.join();
    for (size_t t = 0; t < parts; ++t)
        if (codes[t] != 0) throw StError(codes[t], errors[t]);
}

void write_full(int fd, const void* src, size_t n) {
    const auto* p = static_cast<const uint8_t*>(src);
    while (n > 0) {
        const ssize_t r = ::write(fd, p, n);
        if (r < 0) {
            if (errno == EINTR) continue;
            io_error("write failed");
        }
        p += r;
        n -= static_cast<size_t>(r);
    }
}

int element_bytes(const std::string& dtype) {  // Entry.bytesPerElement, SafeTensors.kt:23-30
    if (dtype == "F32" || dtype == "I32" || dtype == "U32") return 4;
    if (dtype == "F16" || dtype == "BF16" || dtype == "I16" || dtype == "U16") return 2;
    if (dtype == "F64" || dtype == "I64" || dtype == "U64") return 8;
    if (dtype == "I8" || dtype == "U8" || dtype == "BOOL") return 1;
    return 0;
}

// ------------------------------------------------------------------ conversion to float32
enum Conv : int32_t { kF16 = 1, kBF16, kF64, kI8, kU8, kI16, kI32, kI64 };

int conv_of(const std::string& dtype) {  // SafeTensors.convert, SafeTensors.kt:136-170
    if (dtype == "F16") return kF16;
    if (dtype == "BF16") return kBF16;
    if (dtype == "F64") return kF64;
    if (dtype == "I8") return kI8;
    if (dtype == "U8" || dtype == "BOOL") return kU8;
    if (dtype == "I16") return kI16;
    if (dtype == "I32") return kI32;
    if (dtype == "I64") return kI64;
    return 0;
}

// IEEE binary16 bits -> binary32 bits, exact for every input (infinities and
// NaNs keep sign and payload; subnormals are renormalised).
__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
    const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0x1Fu) {
        bits = (sign << 31) | 0x7F800000u | (man << 13);
    } else if (exp != 0u) {
        bits = (sign << 31) | ((exp + 112u) << 23) | (man << 13);  // rebias 15 -> 127
    } else if (man == 0u) {
        bits = sign << 31;
    } else {
        // man * 2^-24 = 1.f * 2^(lead - 24) with `lead` the top set bit of man (0..9)
        const int lead = 31 - __clz(man);
        bits = (sign << 31) | (static_cast<uint32_t>(lead - 24 + 127) << 23) | ((man << (23 - lead)) & 0x7FFFFFu);
    }
    return __uint_as_float(bits);
}

__global__ void to_f32_kernel(const uint8_t* __restrict__ src, int32_t conv, int64_t n, float* __restrict__ dst) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v;
        switch (conv) {
            case kF16: v = half_bits_to_float(reinterpret_cast<const uint16_t*>(src)[i]); break;
            case kBF16: v = __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(src)[i]) << 16); break;
            case kF64: v = __double2float_rn(reinterpret_cast<const double*>(src)[i]); break;
            case kI8: v = static_cast<float>(reinterpret_cast<const int8_t*>(src)[i]); break;
            case kU8: v = static_cast<float>(src[i]); break;
            case kI16: v = static_cast<float>(reinterpret_cast<const int16_t*>(src)[i]); break;
            case kI32: v = __int2float_rn(reinterpret_cast<const int32_t*>(src)[i]); break;
            default: v = __ll2float_rn(reinterpret_cast<const long long*>(src)[i]); break;
        }
        dst[i] = v;
    }
}

// Two pinned host buffers (and, for converting reads, two device buffers) with
// an event each, bound to one device.
struct Staging {
    int device = -1;
    uint8_t* host[2] = {nullptr, nullptr};
    uint8_t* dev[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int next = 0;

    void ensure(int dev_index, bool need_dev) {
        if (device != dev_index) release();
        cuda_check(cudaSetDevice(dev_index), "cudaSetDevice");
        device = dev_index;
        for (int b = 0; b < 2; ++b) {
            if (!done[b]) cuda_check(cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming), "cudaEventCreate");
            if (!host[b])
                cuda_check(cudaHostAlloc(reinterpret_cast<void**>(&host[b]), kChunk, cudaHostAllocPortable),
                           "cudaHostAlloc(staging)");
            if (need_dev && !dev[b]) cuda_check(cudaMalloc(reinterpret_cast<void**>(&dev[b]), kChunk), "cudaMalloc(staging)");
        }
    }
    // The buffer to fill next, once the work that last used it has finished.
    int take() {
        const int b = next;
        next ^= 1;
        cuda_check(cudaEventSynchronize(done[b]), "staging wait");
        return b;
    }
    void release() {
        if (device < 0) return;
        cudaSetDevice(device);
        for (int b = 0; b < 2; ++b) {
            if (done[b]) {
                cudaEventSynchronize(done[b]);
                cudaEventDestroy(done[b]);
            }
            if (host[b]) cudaFreeHost(host[b]);
            if (dev[b]) cudaFree(dev[b]);
            done[b] = nullptr;
            host[b] = dev[b] = nullptr;
        }
        device = -1;
        next = 0;
    }
    ~Staging() { release(); }
};

struct Entry {
    std::string name, dtype;
    std::vector<int64_t> shape;
    int64_t offset = 0, bytes = 0;
};

template <typename F>
kt_status guarded(F&& body) {
    try {
        body();
        return KT_OK;
    } catch (const StError& e) {
        kt::set_error(e.what());
        return e.status;
    } catch (const std::bad_alloc&) {
        kt::set_error("host allocation failed");
        return KT_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        kt::set_error(e.what());
        return KT_ERR_INVALID_ARGUMENT;
    }
}

// JSON string of the reference's writer (SafeTensors.jsonString, SafeTensors.kt:251-264).
void json_string(std::string& out, const char* text) {
    out.push_back('"');
    for (const char* p = text; *p; ++p) {
        const unsigned char c = static_cast<unsigned char>(*p);
        switch (c) {
            case '"': out += "\\\""; break;
            case '\\': out += "\\\\"; break;
            case '\n': out += "\\n"; break;
            case '\r': out += "\\r"; break;
            case '\t': out += "\\t"; break;
            default:
                if (c < 0x20) {
                    char buf[8];
                    std::snprintf(buf, sizeof buf, "\\u%04x", c);
                    out += buf;
                } else {
                    out.push_back(static_cast<char>(c));
                }
        }
    }
    out.push_back('"');
}

}  // namespace

struct kt_stfile {
    std::string path;
    int fd = -1;
    int64_t file_bytes = 0, data_start = 0;
    std::vector<Entry> entries;
    std::unordered_map<std::string, size_t> by_name;
    std::vector<std::pair<std::string, std::string>> metadata;
    std::mutex staging_mutex;  // one device transfer at a time per file
    Staging staging;

    const Entry& entry(const std::string& name) const {
        auto it = by_name.find(name);
        if (it == by_name.end()) bad("No tensor named '" + name + "' in " + path);
        return entries[it->second];
    }
    ~kt_stfile() {
        staging.release();
        if (fd >= 0) ::close(fd);
    }
};

namespace {

void parse_header(kt_stfile* f) {
    uint8_t size_bytes[8];
    pread_full(f->fd, size_bytes, 8, 0);
    int64_t header = 0;
    for (int k = 7; k >= 0; --k) header = (header << 8) | size_bytes[k];
    if (header < 1 || header > kMaxHeader)
        bad("Invalid safetensors header size " + std::to_string(header) + " in " + f->path);
    if (8 + header > f->file_bytes) {
        errno = EIO;
        io_error("header of " + f->path + " runs past the end of the file");
    }
    std::string text(static_cast<size_t>(header), '\0');
    pread_full(f->fd, &text[0], text.size(), 8);
    f->data_start = 8 + header;
    const JValue doc = JsonReader(text.data(), text.size()).document();
    if (doc.kind != JValue::Obj) bad("safetensors header of " + f->path + " is not a JSON object");
    for (const auto& kv : doc.obj) {
        const std::string& name = kv.first;
        const JValue& body = kv.second;
        if (body.kind != JValue::Obj) continue;
        if (name == "__metadata__") {
            for (const auto& m : body.obj) {
                bool replaced = false;
                for (auto& have : f->metadata)
                    if (have.first == m.first) {
                        have.second = as_text(m.second);
                        replaced = true;
                    }
                if (!replaced) f->metadata.emplace_back(m.first, as_text(m.second));
            }
            continue;
        }
        const JValue* dtype = nullptr;
        const JValue* shape = nullptr;
        const JValue* offsets = nullptr;
        for (const auto& m : body.obj) {
            if (m.first == "dtype") dtype = &m.second;
            else if (m.first == "shape") shape = &m.second;
            else if (m.first == "data_offsets") offsets = &m.second;
        }
        if (!dtype || dtype->kind != JValue::Str) bad("Tensor " + name + " has no dtype");
        Entry e;
        e.name = name;
        e.dtype = dtype->s;
        if (e.dtype.size() >= 8) bad("Tensor " + name + " has dtype '" + e.dtype + "'");
        if (shape && shape->kind == JValue::Arr) {
            if (shape->arr.size() > static_cast<size_t>(kMaxRank))
                bad("Tensor " + name + " has more than " + std::to_string(kMaxRank) + " dimensions");
            for (const auto& d : shape->arr) {
                const int64_t dim = as_long(d, "shape of " + name);
                if (dim < 0 || dim > INT32_MAX)
                    bad("Tensor " + name + " has dimension " + std::to_string(dim) + " outside [0, 2^31)");
                e.shape.push_back(static_cast<int32_t>(dim));
            }
        }
        if (!offsets || offsets->kind != JValue::Arr || offsets->arr.size() < 2)
            bad("Tensor " + name + " has no data_offsets");
        const int64_t start = as_long(offsets->arr[0], "data_offsets of " + name);
        const int64_t end = as_long(offsets->arr[1], "data_offsets of " + name);
        // The reference checks end >= start and the end against the file size;
        // a negative start is refused as well.
        if (start < 0 || end < start || end > f->file_bytes - f->data_start)  // no signed overflow
            bad("Tensor " + name + " data range [" + std::to_string(start) + ", " + std::to_string(end) +
                ") exceeds file " + std::to_string(f->file_bytes));
        e.offset = start;
        e.bytes = end - start;
        auto it = f->by_name.find(name);
        if (it != f->by_name.end()) {
            f->entries[it->second] = std::move(e);
        } else {
            f->by_name.emplace(name, f->entries.size());
            f->entries.push_back(std::move(e));
        }
    }
}

// Entry bytes [0, e.bytes) to device memory: raw bytes to `dst`, or float32
// converted by `conv` to `fdst`.
void to_device(kt_stfile* f, kt_ctx* ctx, const Entry& e, uint8_t* dst, int conv, float* fdst, cudaStream_t s) {
    std::lock_guard<std::mutex> lock(f->staging_mutex);
    Staging& st = f->staging;
    st.ensure(ctx->device, conv != 0);
    const int esize = conv != 0 ? element_bytes(e.dtype) : 1;
    for (int64_t off = 0; off < e.bytes; off += static_cast<int64_t>(kChunk)) {
        const size_t n = static_cast<size_t>(std::min<int64_t>(static_cast<int64_t>(kChunk), e.bytes - off));
        const int b = st.take();
        read_parallel(f->fd, st.host[b], n, f->data_start + e.offset + off);
        if (conv == 0) {
            cuda_check(cudaMemcpyAsync(dst + off, st.host[b], n, cudaMemcpyHostToDevice, s), "copy to device");
        } else {
            cuda_check(cudaMemcpyAsync(st.dev[b], st.host[b], n, cudaMemcpyHostToDevice, s), "copy to device");
            const int64_t count = static_cast<int64_t>(n) / esize;
            const int blocks = static_cast<int>(std::min<int64_t>((count + 255) / 256, 148 * 8));
            to_f32_kernel<<<blocks, 256, 0, s>>>(st.dev[b], conv, count, fdst + off / esize);
            cuda_check(cudaGetLastError(), "conversion launch");
        }
        cuda_check(cudaEventRecord(st.done[b], s), "cudaEventRecord");
    }
}

}  // namespace

extern "C" {

kt_status kt_st_open(const char* path, kt_stfile** out) {
    if (!path || !out) {
        kt::set_error("NULL argument");
        return KT_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    kt_stfile* f = new (std::nothrow) kt_stfile();
    if (!f) {
        kt::set_error("host allocation failed");
        return KT_ERR_OUT_OF_MEMORY;
    }
    const kt_status st = guarded([&] {
        f->path = path;
        f->fd = ::open(path, O_RDONLY | O_CLOEXEC);
        if (f->fd < 0) io_error(std::string(path));
        struct stat sb;
        if (::fstat(f->fd, &sb) != 0) io_error(std::string(path));
        f->file_bytes = static_cast<int64_t>(sb.st_size);
        parse_header(f);
    });
    if (st != KT_OK) {
        delete f;
        return st;
    }
    *out = f;
    return KT_OK;
}

kt_status kt_st_close(kt_stfile* f) {
    delete f;
    return KT_OK;
}

int32_t kt_st_tensor_count(const kt_stfile* f) { return f ? static_cast<int32_t>(f->entries.size()) : 0; }

const char* kt_st_tensor_name(const kt_stfile* f, int32_t index) {
    if (!f || index < 0 || index >= static_cast<int32_t>(f->entries.size())) return nullptr;
    return f->entries[static_cast<size_t>(index)].name.c_str();
}

kt_status kt_st_entry(const kt_stfile* f, const char* name, kt_st_entry_info* out) {
    if (!f || !name || !out) {
        kt::set_error("NULL argument");
        return KT_ERR_INVALID_ARGUMENT;
    }
    return guarded([&] {
        const Entry& e = f->entry(name);
        std::memset(out, 0, sizeof(*out));
        std::memcpy(out->dtype, e.dtype.c_str(), e.dtype.size() + 1);
        out->rank = static_cast<int32_t>(e.shape.size());
        for (size_t d = 0; d < e.shape.size(); ++d) out->shape[d] = e.shape[d];
        out->offset = e.offset;
        out->bytes = e.bytes;
    });
}

int32_t kt_st_metadata_count(const kt_stfile* f) { return f ? static_cast<int32_t>(f->metadata.size()) : 0; }

kt_status kt_st_metadata_at(const kt_stfile* f, int32_t index, const char** key, const char** value) {
    if (!f || !key || !value || index < 0 || index >= static_cast<int32_t>(f->metadata.size())) {
        kt::set_error("metadata index out of range");
        return KT_ERR_INVALID_ARGUMENT;
    }
    *key = f->metadata[static_cast<size_t>(index)].first.c_str();
    *value = f->metadata[static_cast<size_t>(index)].second.c_str();
    return KT_OK;
}

kt_status kt_st_read_raw(kt_stfile* f, const char* name, void* dst, int64_t capacity) {
    if (!f || !name || (!dst && capacity > 0)) {
        kt::set_error("NULL argument");
        return KT_ERR_INVALID_ARGUMENT;
    }
    return guarded([&] {
        const Entry& e = f->entry(name);
        if (e.bytes > capacity)
            bad("Destination too small for " + e.name + ": needs " + std::to_string(e.bytes) + " bytes at 0, has " +
                std::to_string(capacity));
        read_parallel(f->fd, dst, static_cast<size_t>(e.bytes), f->data_start + e.offset);
    });
}

kt_status kt_st_read_raw_device(kt_ctx* ctx, kt_stfile* f, const char* name, void* dst, int64_t capacity,
                                void* stream) {
    if (!ctx || !f || !name || (!dst && capacity > 0)) {
        kt::set_error("NULL argument");
        return KT_ERR_INVALID_ARGUMENT;
    }
    return guarded([&] {
        const Entry& e = f->entry(name);
        if (e.bytes > capacity)
            bad("Destination too small for " + e.name + ": needs " + std::to_string(e.bytes) + " bytes at 0, has " +
                std::to_string(capacity));
        to_device(f, ctx, e, static_cast<uint8_t*>(dst), 0, nullptr, static_cast<cudaStream_t>(stream));
    });
}

kt_status kt_st_read_f32_device(kt_ctx* ctx, kt_stfile* f, const char* name, float* dst, int64_t capacity,
                                void* stream) {
    if (!ctx || !f || !name || (!dst && capacity > 0)) {
        kt::set_error("NULL argument");
        return KT_ERR_INVALID_ARGUMENT;
    }
    return guarded([&] {
        const Entry& e = f->entry(name);
        const int esize = element_bytes(e.dtype);
        if (esize == 0) bad("Unsupported safetensors dtype '" + e.dtype + "' for tensor " + e.name);
        int64_t count = 1;
        for (int64_t d : e.shape) count *= d;
        if (count > INT32_MAX)
            bad("Tensor " + e.name + " has " + std::to_string(count) + " elements, more than a FloatArray can hold");
        if (count < 0 || count > capacity)
            bad("Destination too small for " + e.name + ": needs " + std::to_string(count) + " elements at 0, has " +
                std::to_string(capacity));
        if (e.bytes != count * esize)
            bad("Tensor " + e.name + " has " + std::to_string(e.bytes) + " bytes for " + std::to_string(count) + " " +
                e.dtype + " elements");
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (e.dtype == "F32") {
            to_device(f, ctx, e, reinterpret_cast<uint8_t*>(dst), 0, nullptr, s);
            return;
        }
        const int conv = conv_of(e.dtype);
        if (conv == 0) bad("Unsupported safetensors dtype '" + e.dtype + "'");
        to_device(f, ctx, e, nullptr, conv, dst, s);
    });
}

kt_status kt_st_write(kt_ctx* ctx, const char* path, const kt_st_tensor* tensors, int32_t count,
                      const char* const* meta_keys, const char* const* meta_values, int32_t meta_count,
                      void* stream) {
    if (!path || count < 0 || meta_count < 0 || (count > 0 && !tensors) ||
        (meta_count > 0 && (!meta_keys || !meta_values))) {
        kt::set_error("NULL argument");
        return KT_ERR_INVALID_ARGUMENT;
    }
    int fd = -1;
    const kt_status st = guarded([&] {
        bool any_device = false;
        for (int32_t t = 0; t < count; ++t) {
            const kt_st_tensor& x = tensors[t];
            if (!x.name || !x.dtype) bad("tensor " + std::to_string(t) + " has no name or dtype");
            if (x.rank < 0 || x.rank > kMaxRank || (x.rank > 0 && !x.shape))
                bad("tensor " + std::string(x.name) + " has an invalid shape");
            if (x.bytes < 0 || (x.bytes > 0 && !x.data)) bad("tensor " + std::string(x.name) + " has no data");
            any_device = any_device || (x.on_device && x.bytes > 0);
        }
        if (any_device && !ctx) bad("device tensors need a context");
        for (int32_t k = 0; k < meta_count; ++k)
            if (!meta_keys[k] || !meta_values[k]) bad("NULL metadata key or value");

        std::string header = "{";
        bool first = true;
        if (meta_count > 0) {
            header += "\"__metadata__\":{";
            for (int32_t k = 0; k < meta_count; ++k) {
                if (k) header.push_back(',');
                json_string(header, meta_keys[k]);
                header.push_back(':');
                json_string(header, meta_values[k]);
            }
            header += "}";
            first = false;
        }
        int64_t offset = 0;
        for (int32_t t = 0; t < count; ++t) {
            const kt_st_tensor& x = tensors[t];
            if (!first) header.push_back(',');
            first = false;
            json_string(header, x.name);
            header += ":{\"dtype\":\"";
            header += x.dtype;
            header += "\",\"shape\":[";
            for (int32_t d = 0; d < x.rank; ++d) {
                if (d) header.push_back(',');
                header += std::to_string(x.shape[d]);
            }
            header += "],\"data_offsets\":[" + std::to_string(offset) + "," + std::to_string(offset + x.bytes) + "]}";
            offset += x.bytes;
        }
        header.push_back('}');
        const size_t padding = (8 - header.size() % 8) % 8;
        header.append(padding, ' ');
        uint8_t size_bytes[8];
        uint64_t hs = header.size();
        for (int k = 0; k < 8; ++k) size_bytes[k] = static_cast<uint8_t>(hs >> (8 * k));

        fd = ::open(path, O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
        if (fd < 0) io_error(std::string(path));
        write_full(fd, size_bytes, 8);
        write_full(fd, header.data(), header.size());

        Staging staging;
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (any_device) staging.ensure(ctx->device, false);
        for (int32_t t = 0; t < count; ++t) {
            const kt_st_tensor& x = tensors[t];
            if (x.bytes == 0) continue;
            if (!x.on_device) {
                write_full(fd, x.data, static_cast<size_t>(x.bytes));
                continue;
            }
            // device -> pinned chunk i+1 while chunk i goes to the file
            const auto* src = static_cast<const uint8_t*>(x.data);
            const int64_t chunks = (x.bytes + static_cast<int64_t>(kChunk) - 1) / static_cast<int64_t>(kChunk);
            auto issue = [&](int64_t i) {
                const int b = static_cast<int>(i & 1);
                const size_t n = static_cast<size_t>(
                    std::min<int64_t>(static_cast<int64_t>(kChunk), x.bytes - i * static_cast<int64_t>(kChunk)));
                cuda_check(cudaMemcpyAsync(staging.host[b], src + i * static_cast<int64_t>(kChunk), n,
                                           cudaMemcpyDeviceToHost, s),
                           "copy from device");
                cuda_check(cudaEventRecord(staging.done[b], s), "cudaEventRecord");
            };
            issue(0);
            for (int64_t i = 0; i < chunks; ++i) {
                if (i + 1 < chunks) issue(i + 1);
                const int b = static_cast<int>(i & 1);
                cuda_check(cudaEventSynchronize(staging.done[b]), "copy from device");
                const size_t n = static_cast<size_t>(
                    std::min<int64_t>(static_cast<int64_t>(kChunk), x.bytes - i * static_cast<int64_t>(kChunk)));
                write_full(fd, staging.host[b], n);
            }
        }
        if (::close(fd) != 0) {
            fd = -1;
            io_error(std::string(path));
        }
        fd = -1;
    });
    if (fd >= 0) ::close(fd);
    return st;
}

}  // extern "C"
