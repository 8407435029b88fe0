// GGUF container reader (host side): the directory parser and tensor payload
// reads that feed tc_cuda_weight_upload.
//
// Restates the acceptance rules of the reference parser
// (native/core/gguf_directory.hpp:199-271, read_directory; split sets :273-304,
// validate_split_set) in this library's own structure: a buffered pread
// cursor with the same parse limits, the same checks in the same order and
// the same error texts ("gguf_invalid: <reason>"), so a file the reference
// rejects is rejected here with the same reason.  GGML type table:
// gguf_directory.hpp:19-30.  The caller's file stays open for payload reads
// (pread at file_offset + row * row_bytes), as the reference's streaming
// loaders read it (gguf_packed_bank.cpp:374-517).
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <limits>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_set>
#include <vector>

#include "../../include/turbocider_cuda.h"
#include "tc_internal.h"

namespace {

struct GgmlType {
    uint32_t id, elements, bytes;
};
// On-disk GGML type ids with (elements, bytes) per block.
constexpr GgmlType kGgmlTypes[] = {{0, 1, 4},    {1, 1, 2},    {2, 32, 18},   {3, 32, 20},
                                   {6, 32, 22},  {7, 32, 24},  {8, 32, 34},   {12, 256, 144},
                                   {13, 256, 176}, {14, 256, 210}, {30, 1, 2}};

[[noreturn]] void invalid(const std::string &reason) { throw std::invalid_argument("gguf_invalid: " + reason); }
void require(bool ok, const char *reason) {
    if (!ok) invalid(reason);
}
uint64_t add_checked(uint64_t a, uint64_t b) {
    require(b <= UINT64_MAX - a, "integer addition overflow");
    return a + b;
}
uint64_t mul_checked(uint64_t a, uint64_t b) {
    require(!a || b <= UINT64_MAX / a, "integer multiplication overflow");
    return a * b;
}
const GgmlType &ggml_type(uint32_t id) {
    for (const auto &t : kGgmlTypes)
        if (t.id == id) return t;
    throw std::invalid_argument("gguf_type_unsupported: " + std::to_string(id));
}

struct Limits {
    uint64_t tensors = 65536, metadata_entries = 65536;
    uint64_t directory_bytes = 64ull << 20, retained_bytes = 32ull << 20;
    uint64_t string_bytes = 1ull << 20, array_elements = 1ull << 20;
    uint32_t max_rank = 4, max_array_depth = 4;
};

struct Meta {
    std::string key, text;
    uint32_t type = 0, element_type = 0;
    uint64_t count = 0, u = 0;
    int64_t i = 0;
    double f = 0;
};
struct Tensor {
    std::string name;
    uint32_t type = 0;
    std::vector<uint64_t> dims;   // dims[0] is the contiguous (column) extent
    uint64_t relative = 0, offset = 0, bytes = 0, elements = 0;
};

// Sequential reader over the directory region: every read is bounded by the
// file size and the directory byte limit, and each retained byte (strings,
// table entries) is charged against the retained-metadata limit.
class Cursor {
  public:
    Cursor(int fd, uint64_t size, const Limits &lim) : fd_(fd), size_(size), lim_(lim) {
        require(fd >= 0 && size <= uint64_t(std::numeric_limits<off_t>::max()), "invalid fd/size");
    }
    uint64_t pos() const { return pos_; }
    uint64_t retained() const { return retained_; }
    void charge(uint64_t n) {
        retained_ = add_checked(retained_, n);
        require(retained_ <= lim_.retained_bytes, "retained metadata limit");
    }
    void advance(uint64_t n) {
        require(pos_ <= size_ && n <= size_ - pos_, "truncated directory");
        require(pos_ <= lim_.directory_bytes && n <= lim_.directory_bytes - pos_, "directory byte limit");
        pos_ += n;
    }
    void bytes(void *dst, uint64_t n) {
        const uint64_t at = pos_;
        advance(n);
        auto *out = static_cast<uint8_t *>(dst);
        uint64_t got = 0;
        while (got < n) {
            const uint64_t p = at + got;
            if (p >= buf_at_ && p < buf_at_ + buf_len_) {   // served from the buffer
                const uint64_t take = std::min<uint64_t>(n - got, buf_at_ + buf_len_ - p);
                std::memcpy(out + got, buf_.data() + (p - buf_at_), size_t(take));
                got += take;
                continue;
            }
            if (n - got >= buf_.size()) {                    // large read: straight into dst
                const ssize_t r = ::pread(fd_, out + got, size_t(std::min<uint64_t>(n - got, 1ull << 20)), off_t(p));
                if (r < 0 && errno == EINTR) continue;
                require(r > 0, "directory read failed or source changed");
                got += uint64_t(r);
                continue;
            }
            const uint64_t end = std::min(size_, lim_.directory_bytes);
            const ssize_t r = ::pread(fd_, buf_.data(), size_t(std::min<uint64_t>(buf_.size(), end - p)), off_t(p));
            if (r < 0 && errno == EINTR) continue;
            require(r > 0, "directory read failed or source changed");
            buf_at_ = p;
            buf_len_ = uint64_t(r);
        }
    }
    uint64_t uint(uint32_t width) {
        uint8_t b[8] = {};
        require(width && width <= 8, "invalid scalar width");
        bytes(b, width);
        uint64_t v = 0;
        for (uint32_t k = 0; k < width; ++k) v |= uint64_t(b[k]) << (8 * k);
        return v;
    }
    std::string str(bool keep) {
        const uint64_t n = uint(8);
        require(n <= lim_.string_bytes, "string byte limit");
        if (!keep) {
            advance(n);
            return {};
        }
        charge(add_checked(n, 1));
        require(n <= size_ - pos_ && n <= lim_.directory_bytes - pos_, "truncated string");
        std::string s(size_t(n), '\0');
        bytes(s.data(), n);
        return s;
    }
    // One metadata value of GGUF type `type`; arrays are walked (nested up to
    // max_array_depth) but not retained.
    void value(uint32_t type, Meta *m, uint32_t depth = 0) {
        if (type == 8) {
            std::string s = str(m != nullptr);
            if (m) m->text = std::move(s);
            return;
        }
        if (type == 9) {
            require(depth < lim_.max_array_depth, "nested array depth limit");
            const uint32_t elem = uint32_t(uint(4));
            const uint64_t count = uint(8);
            require(count <= lim_.array_elements, "array element limit");
            require(elem <= 12, "invalid array element type");
            if (m) {
                m->element_type = elem;
                m->count = count;
            }
            if (elem == 7 || elem == 8 || elem == 9)
                for (uint64_t k = 0; k < count; ++k) value(elem, nullptr, depth + 1);
            else
                advance(mul_checked(count, width(elem)));
            return;
        }
        const uint32_t w = width(type);
        const uint64_t raw = uint(w);
        if (type == 7) require(raw <= 1, "invalid boolean");
        if (!m) return;
        m->u = raw;
        if (type == 1 || type == 3 || type == 5 || type == 11) {   // signed: sign-extend
            const uint64_t sign = uint64_t(1) << (8 * w - 1);
            m->i = int64_t(w == 8 || !(raw & sign) ? raw : raw | (UINT64_MAX << (8 * w)));
        }
        if (type == 6) {
            float f;
            const uint32_t r32 = uint32_t(raw);
            std::memcpy(&f, &r32, 4);
            m->f = f;
        }
        if (type == 12) std::memcpy(&m->f, &raw, 8);
    }

  private:
    static uint32_t width(uint32_t type) {
        switch (type) {
        case 0: case 1: case 7: return 1;
        case 2: case 3: return 2;
        case 4: case 5: case 6: return 4;
        case 10: case 11: case 12: return 8;
        default: invalid("invalid metadata scalar type");
        }
    }
    int fd_;
    uint64_t size_, pos_ = 0, retained_ = 0;
    const Limits &lim_;
    std::vector<uint8_t> buf_ = std::vector<uint8_t>(64 * 1024);
    uint64_t buf_at_ = 0, buf_len_ = 0;
};

}  // namespace

struct tc_gguf {
    int fd = -1;
    uint32_t version = 0, alignment = 32;
    uint64_t file_bytes = 0, directory_end = 0, data_offset = 0, retained = 0;
    std::vector<Meta> meta;
    std::vector<Tensor> tensors;
    ~tc_gguf() {
        if (fd >= 0) ::close(fd);
    }
    const Meta *find_meta(const char *key) const {
        for (const auto &m : meta)
            if (m.key == key) return &m;
        return nullptr;
    }
};

namespace {

// Parse the directory of an open file (gguf_directory.hpp:199-271).
void parse(tc_gguf &g, const Limits &lim) {
    Cursor in(g.fd, g.file_bytes, lim);
    require(lim.max_rank <= 8 && lim.max_array_depth <= 8, "unsafe parser limits");
    require(in.uint(4) == 0x46554747u, "invalid GGUF magic/endian");
    g.version = uint32_t(in.uint(4));
    require(g.version == 2 || g.version == 3, "unsupported GGUF version");
    const uint64_t n_tensors = in.uint(8), n_meta = in.uint(8);
    require(n_tensors && n_tensors <= lim.tensors && n_tensors <= g.file_bytes / 24, "tensor count limit");
    require(n_meta <= lim.metadata_entries && n_meta <= g.file_bytes / 12, "metadata count limit");
    in.charge(mul_checked(n_tensors, sizeof(Tensor) + 256));
    in.charge(mul_checked(n_meta, sizeof(Meta) + 128));
    g.meta.reserve(size_t(n_meta));
    g.tensors.reserve(size_t(n_tensors));
    std::unordered_set<std::string> seen;
    for (uint64_t k = 0; k < n_meta; ++k) {
        Meta m;
        m.key = in.str(true);
        require(!m.key.empty() && m.key.find('\0') == std::string::npos, "invalid metadata key");
        in.charge(m.key.size() + 1);
        require(seen.insert(m.key).second, "duplicate metadata key");
        m.type = uint32_t(in.uint(4));
        in.value(m.type, &m);
        g.meta.push_back(std::move(m));
    }
    if (const Meta *a = g.find_meta("general.alignment")) {
        require(a->type == 4, "alignment must be uint32");
        require(a->u && a->u <= (1u << 20) && !(a->u & (a->u - 1)), "invalid alignment");
        g.alignment = uint32_t(a->u);
    }
    seen.clear();
    for (uint64_t k = 0; k < n_tensors; ++k) {
        Tensor t;
        t.name = in.str(true);
        require(!t.name.empty() && t.name.find('\0') == std::string::npos, "invalid tensor name");
        in.charge(t.name.size() + 1);
        require(seen.insert(t.name).second, "duplicate tensor name");
        const uint32_t rank = uint32_t(in.uint(4));
        require(rank && rank <= lim.max_rank, "invalid tensor rank");
        t.elements = 1;
        for (uint32_t d = 0; d < rank; ++d) {
            const uint64_t dim = in.uint(8);
            require(dim && dim <= uint64_t(INT32_MAX), "invalid tensor dimension");
            t.elements = mul_checked(t.elements, dim);
            t.dims.push_back(dim);
        }
        t.type = uint32_t(in.uint(4));
        const GgmlType &gt = ggml_type(t.type);
        require(t.dims[0] % gt.elements == 0, "continuous dimension is not block aligned");
        t.bytes = mul_checked(t.elements / gt.elements, gt.bytes);
        t.relative = in.uint(8);
        require(t.relative % g.alignment == 0, "unaligned tensor offset");
        g.tensors.push_back(std::move(t));
    }
    g.directory_end = in.pos();
    const uint64_t mask = g.alignment - 1;
    g.data_offset = add_checked(g.directory_end, mask) & ~mask;
    require(g.data_offset <= g.file_bytes, "missing aligned tensor data");
    std::vector<std::pair<uint64_t, uint64_t>> spans;
    spans.reserve(g.tensors.size());
    for (auto &t : g.tensors) {
        t.offset = add_checked(g.data_offset, t.relative);
        require(t.offset <= g.file_bytes && t.bytes <= g.file_bytes - t.offset, "tensor payload out of file bounds");
        spans.emplace_back(t.offset, add_checked(t.offset, t.bytes));
    }
    std::sort(spans.begin(), spans.end());
    for (size_t k = 1; k < spans.size(); ++k) require(spans[k].first >= spans[k - 1].second, "overlapping tensor payloads");
    g.retained = in.retained();
}

int fail_msg(const std::string &m) {
    tc::set_last_error(m);
    return TC_CUDA_FAIL;
}
int ok() {
    tc::set_last_error("");
    return TC_CUDA_OK;
}

}  // namespace

extern "C" {

int tc_gguf_open(const char *path, const char *limit, tc_gguf **out) {
    if (!path || !out) return fail_msg("null argument");
    *out = nullptr;
    try {
        auto g = std::make_unique<tc_gguf>();
        g->fd = ::open(path, O_RDONLY | O_CLOEXEC);
        struct stat st {};
        require(g->fd >= 0 && ::fstat(g->fd, &st) == 0 && st.st_size >= 0, "cannot open file");
        g->file_bytes = uint64_t(st.st_size);
        Limits lim;
        if (limit && *limit) {   // test hook: shrink one parse limit
            const std::string l(limit);
            if (l == "retained") lim.retained_bytes = 1;
            else if (l == "directory") lim.directory_bytes = 24;
            else if (l == "string") lim.string_bytes = 1;
            else if (l == "count") lim.tensors = 1;
            else if (l == "array") lim.array_elements = 1;
            else throw std::invalid_argument("unknown test limit");
        }
        parse(*g, lim);
        *out = g.release();
        return ok();
    } catch (const std::exception &e) {
        return fail_msg(e.what());
    }
}

void tc_gguf_close(tc_gguf *g) { delete g; }

int tc_gguf_info(const tc_gguf *g, uint32_t *version, uint32_t *alignment, uint64_t *n_tensors,
                 uint64_t *data_offset, uint64_t *n_metadata) {
    if (!g) return fail_msg("null file");
    if (version) *version = g->version;
    if (alignment) *alignment = g->alignment;
    if (n_tensors) *n_tensors = g->tensors.size();
    if (data_offset) *data_offset = g->data_offset;
    if (n_metadata) *n_metadata = g->meta.size();
    return ok();
}

int tc_gguf_tensor(const tc_gguf *g, uint64_t index, char *name, uint64_t name_cap, uint32_t *ggml_type,
                   uint32_t *rank, uint64_t *dims, uint64_t *file_offset, uint64_t *bytes) {
    if (!g) return fail_msg("null file");
    if (index >= g->tensors.size()) return fail_msg("tensor index out of range");
    const Tensor &t = g->tensors[size_t(index)];
    if (name) {
        if (name_cap < t.name.size() + 1) return fail_msg("name buffer too small");
        std::memcpy(name, t.name.c_str(), t.name.size() + 1);
    }
    if (ggml_type) *ggml_type = t.type;
    if (rank) *rank = uint32_t(t.dims.size());
    if (dims)
        for (size_t d = 0; d < 4; ++d) dims[d] = d < t.dims.size() ? t.dims[d] : 1;
    if (file_offset) *file_offset = t.offset;
    if (bytes) *bytes = t.bytes;
    return ok();
}

int tc_gguf_find(const tc_gguf *g, const char *name, uint64_t *index) {
    if (!g || !name || !index) return fail_msg("null argument");
    for (size_t k = 0; k < g->tensors.size(); ++k)
        if (g->tensors[k].name == name) {
            *index = k;
            return ok();
        }
    return fail_msg(std::string("gguf_tensor_missing: ") + name);
}

int tc_gguf_meta(const tc_gguf *g, const char *key, uint32_t *type, uint64_t *u, int64_t *i, double *f, char *text,
                 uint64_t text_cap, uint64_t *array_count) {
    if (!g || !key) return fail_msg("null argument");
    const Meta *m = g->find_meta(key);
    if (!m) return fail_msg(std::string("gguf_metadata_missing: ") + key);
    if (type) *type = m->type;
    if (u) *u = m->u;
    if (i) *i = m->i;
    if (f) *f = m->f;
    if (array_count) *array_count = m->count;
    if (text && m->type == 8) {
        if (text_cap < m->text.size() + 1) return fail_msg("text buffer too small");
        std::memcpy(text, m->text.c_str(), m->text.size() + 1);
    }
    return ok();
}

int tc_gguf_read(const tc_gguf *g, uint64_t index, uint64_t row_begin, uint64_t rows, void *dst, uint64_t dst_bytes,
                 const volatile int32_t *cancel) {
    if (!g || (!dst && rows)) return fail_msg("null argument");
    if (index >= g->tensors.size()) return fail_msg("tensor index out of range");
    const Tensor &t = g->tensors[size_t(index)];
    const GgmlType &gt = ggml_type(t.type);
    const uint64_t total_rows = t.elements / t.dims[0];
    const uint64_t row_bytes = t.dims[0] / gt.elements * gt.bytes;
    if (row_begin > total_rows || rows > total_rows - row_begin) return fail_msg("row range out of bounds");
    const uint64_t n = rows * row_bytes;
    if (dst_bytes < n) return fail_msg("destination too small");
    auto *out = static_cast<uint8_t *>(dst);
    uint64_t got = 0;
    const uint64_t at = t.offset + row_begin * row_bytes;
    while (got < n) {
        // the caller's cancel flag is polled between reads of at most 8 MiB
        if (cancel && *cancel) {
            tc::set_last_error("generation cancelled");
            return TC_CUDA_CANCELLED;
        }
        const ssize_t r = ::pread(g->fd, out + got, size_t(std::min<uint64_t>(n - got, 8ull << 20)), off_t(at + got));
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) return fail_msg("gguf_invalid: payload read failed or source changed");
        got += uint64_t(r);
    }
    return ok();
}

// Split sets (gguf_directory.hpp:273-304): every shard carries split.no /
// split.count / split.tensors.count and one architecture; numbers are unique
// and complete, tensor names unique across shards, and their total matches.
int tc_gguf_validate_split(const tc_gguf *const *shards, uint32_t n) {
    try {
        require(shards && n && n <= 64, "empty/excessive split set");
        Limits lim;
        uint64_t tensor_total = 0, retained_total = 0;
        for (uint32_t s = 0; s < n; ++s) {
            require(shards[s] != nullptr, "empty/excessive split set");
            tensor_total = add_checked(tensor_total, shards[s]->tensors.size());
            retained_total = add_checked(retained_total, shards[s]->retained);
        }
        require(tensor_total <= lim.tensors && retained_total <= lim.retained_bytes, "aggregate split metadata limit");
        std::unordered_set<uint64_t> numbers;
        std::unordered_set<std::string> names;
        std::string arch;
        bool have_arch = false;
        uint64_t count = 0;
        for (uint32_t s = 0; s < n; ++s) {
            const tc_gguf &g = *shards[s];
            const Meta *no = g.find_meta("split.no"), *total = g.find_meta("split.count");
            const Meta *tensors = g.find_meta("split.tensors.count");
            if (n == 1 && !no && !total && !tensors) return ok();
            require(no && total && tensors && no->type == 2 && total->type == 2 &&
                        (tensors->type == 5 || tensors->type == 10),
                    "invalid/missing split metadata");
            require(total->u == n && no->u < n, "missing split shard or invalid split number");
            require(numbers.insert(no->u).second, "duplicate split number");
            require(tensors->type != 5 || tensors->i >= 0, "negative split tensor count");
            if (!count) count = tensors->u;
            require(count && tensors->u == count, "inconsistent split tensor count");
            const Meta *a = g.find_meta("general.architecture");
            require(a && a->type == 8 && !a->text.empty(), "missing split architecture");
            if (!have_arch) {
                arch = a->text;
                have_arch = true;
            }
            require(arch == a->text, "inconsistent split architecture");
            for (const auto &t : g.tensors) require(names.insert(t.name).second, "duplicate split tensor");
        }
        require(names.size() == count, "split tensor count mismatch");
        return ok();
    } catch (const std::exception &e) {
        return fail_msg(e.what());
    }
}

}  // extern "C"
