// Host-side loading for an all-resident MoE: the weight index reader, the
// pinned staging ring behind qg_upload_expert / qg_upload_experts, and the
// route-trace reader. Host code only (no kernels).
//
// * Index (qg_index_*): reads the text index the reference's model loader
//   consumes, COB_QWEN_INDEX_V1 (format and checks as qwen/qwen.c:108-146):
//   a version line, "VERIFIED 1", 3 + 16 + 16 unsigned integers and one int
//   (multipliers, head offsets, head vocabularies > 0, PLE end token), then
//   FILE records (id < 16, byte size, path; the file must exist with exactly
//   that size and is mapped read-only) and TENSOR records (name < 128 chars,
//   file id, offset, bytes, GGML type, four dims; the file must be declared
//   first, the range must lie inside it, the name must be new and the bytes
//   must equal qg_tensor_bytes of the type and dims). Blank lines are allowed;
//   anything else makes the index malformed.
// * Uploads: every expert stays resident, so experts are copied once at load
//   time. A ring of pinned blocks feeds host-to-device copies on the legacy
//   default stream: the host fills block k+1 while block k is in flight, and a
//   block is refilled only after the copy that read it has completed.
//   qg_upload_expert packs one expert's gate|up|down (the reference cache-slot
//   layout); qg_upload_experts moves a list of whole experts of one matrix -
//   all 512 of a layer, or one rank's share under expert parallelism - packing
//   as many experts per block as fit.
// * Route traces (qg_route_trace_*): the QROUTE1 diagnostic stream the
//   reference writes (qwen/qwen.c:87-94 header, :638-646 records): "QROUTE1\n",
//   then per routed layer call three uint32 (layer, target position, tokens),
//   tokens*10 int32 ids and tokens*10 float weights, little-endian.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cctype>
#include <cerrno>
#include <cinttypes>
#include <cstdarg>
#include <climits>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

// ---------------------------------------------------------------- tensor sizes
// Bytes of a GGML tensor whose first dimension is the row length: the row size
// of the type (zero for an unknown type or a ragged last block) times the
// other three dimensions, each non-zero, without overflowing 64 bits.
extern "C" int qg_tensor_bytes(int type, const uint64_t dims[4], uint64_t *bytes) {
    if (!dims || !bytes || dims[0] == 0 || dims[0] > (uint64_t)INT32_MAX) return cudaErrorInvalidValue;
    uint64_t total = nb::row_bytes(type, static_cast<int>(dims[0]));
    if (total == 0) return cudaErrorInvalidValue;
    for (int i = 1; i < 4; i++)
        if (dims[i] == 0 || __builtin_mul_overflow(total, dims[i], &total)) return cudaErrorInvalidValue;
    *bytes = total;
    return cudaSuccess;
}

namespace {

// ---------------------------------------------------------------- staging ring
class StagingRing {
  public:
    static constexpr int kBlocks = 3;

    ~StagingRing() {
        for (Block &b : ring_) {
            if (b.busy) cudaEventSynchronize(b.done);
            if (b.host) cudaFreeHost(b.host);
            if (b.issued) cudaEventDestroy(b.issued);
            if (b.done) cudaEventDestroy(b.done);
        }
    }

    int init(size_t block_bytes) {
        block_bytes_ = block_bytes;
        ring_.resize(kBlocks);
        for (Block &b : ring_) {
            int rc = cudaHostAlloc(reinterpret_cast<void **>(&b.host), block_bytes, cudaHostAllocDefault);
            if (!rc) rc = cudaEventCreate(&b.issued);
            if (!rc) rc = cudaEventCreate(&b.done);
            if (rc) return rc;
        }
        return cudaSuccess;
    }

    size_t block_bytes() const { return block_bytes_; }

    // The next block, once the copy that last read it has completed.
    int next(unsigned char **host, int *slot) {
        const int k = static_cast<int>(turn_++ % ring_.size());
        if (int rc = retire(ring_[k], true)) return rc;
        *host = ring_[k].host;
        *slot = k;
        return cudaSuccess;
    }

    // Copies the first `bytes` of block `slot` to dst on the legacy stream.
    int send(int slot, void *dst, size_t bytes) {
        Block &b = ring_[slot];
        int rc = cudaEventRecord(b.issued, 0);
        if (!rc) rc = cudaMemcpyAsync(dst, b.host, bytes, cudaMemcpyHostToDevice, 0);
        if (!rc) rc = cudaEventRecord(b.done, 0);
        if (!rc) b.busy = true;
        return rc;
    }

    // Device time of every completed copy so far; -1 after a CUDA error.
    double seconds() {
        for (Block &b : ring_)
            if (retire(b, false)) return -1.0;
        return seconds_;
    }

  private:
    struct Block {
        unsigned char *host = nullptr;
        cudaEvent_t issued = nullptr, done = nullptr;
        bool busy = false;
    };

    // Folds a finished copy's duration into the total (waiting for it when asked).
    int retire(Block &b, bool wait) {
        if (!b.busy) return cudaSuccess;
        cudaError_t rc = wait ? cudaEventSynchronize(b.done) : cudaEventQuery(b.done);
        if (rc == cudaErrorNotReady) return cudaSuccess;
        if (rc) return rc;
        float ms = 0.0f;
        if ((rc = cudaEventElapsedTime(&ms, b.issued, b.done))) return rc;
        seconds_ += 1e-3 * ms;
        b.busy = false;
        return cudaSuccess;
    }

    std::vector<Block> ring_;
    size_t block_bytes_ = 0;
    uint64_t turn_ = 0;
    double seconds_ = 0.0;
};

}  // namespace

extern "C" void *qg_upload_create(size_t expert_bytes) {
    if (!expert_bytes) return nullptr;
    auto *ring = new (std::nothrow) StagingRing;
    if (!ring) return nullptr;
    if (ring->init(expert_bytes)) {
        delete ring;
        return nullptr;
    }
    return ring;
}

extern "C" void qg_upload_destroy(void *uploader) { delete static_cast<StagingRing *>(uploader); }

extern "C" int qg_upload_expert(void *uploader, void *dst, const void *gate, size_t gate_bytes, const void *up,
                                size_t up_bytes, const void *down, size_t down_bytes) {
    auto *ring = static_cast<StagingRing *>(uploader);
    size_t total = 0;
    if (!ring || !dst || __builtin_add_overflow(gate_bytes, up_bytes, &total) ||
        __builtin_add_overflow(total, down_bytes, &total) || total > ring->block_bytes())
        return cudaErrorInvalidValue;
    unsigned char *host = nullptr;
    int slot = 0;
    if (int rc = ring->next(&host, &slot)) return rc;
    std::memcpy(host, gate, gate_bytes);
    std::memcpy(host + gate_bytes, up, up_bytes);
    std::memcpy(host + gate_bytes + up_bytes, down, down_bytes);
    return ring->send(slot, dst, total);
}

extern "C" int qg_upload_experts(void *uploader, void *dst, const void *src, size_t expert_bytes, const int *experts,
                                 int count) {
    auto *ring = static_cast<StagingRing *>(uploader);
    if (!ring || !dst || !src || !expert_bytes || count < 1 || expert_bytes > ring->block_bytes())
        return cudaErrorInvalidValue;
    if (experts)
        for (int i = 0; i < count; i++)
            if (experts[i] < 0) return cudaErrorInvalidValue;
    const size_t per_block = ring->block_bytes() / expert_bytes;
    const auto *from = static_cast<const unsigned char *>(src);
    auto *to = static_cast<unsigned char *>(dst);
    for (int i = 0; i < count;) {
        unsigned char *host = nullptr;
        int slot = 0;
        if (int rc = ring->next(&host, &slot)) return rc;
        const int n = static_cast<int>(std::min<size_t>(per_block, static_cast<size_t>(count - i)));
        for (int j = 0; j < n; j++) {
            const size_t e = experts ? static_cast<size_t>(experts[i + j]) : static_cast<size_t>(i + j);
            std::memcpy(host + j * expert_bytes, from + e * expert_bytes, expert_bytes);
        }
        if (int rc = ring->send(slot, to + static_cast<size_t>(i) * expert_bytes, n * expert_bytes)) return rc;
        i += n;
    }
    return cudaSuccess;
}

extern "C" double qg_upload_seconds(void *uploader) {
    auto *ring = static_cast<StagingRing *>(uploader);
    return ring ? ring->seconds() : 0.0;
}

// ---------------------------------------------------------------- weight index
namespace {

constexpr int kIndexFiles = 16;
constexpr size_t kIndexTensors = 1600;

struct IndexTensor {
    int file = -1, type = 0;
    uint64_t offset = 0, bytes = 0, dims[4] = {0, 0, 0, 0};
};

struct MappedFile {
    int fd = -1;
    const unsigned char *data = nullptr;
    uint64_t bytes = 0;
};

struct WeightIndex {
    MappedFile files[kIndexFiles];
    std::unordered_map<std::string, IndexTensor> tensors;
    uint64_t multipliers[3] = {0, 0, 0}, head_offsets[16] = {}, head_vocab[16] = {};
    int ple_eos = 0;

    ~WeightIndex() {
        for (MappedFile &f : files) {
            if (f.data) munmap(const_cast<unsigned char *>(f.data), f.bytes);
            if (f.fd >= 0) close(f.fd);
        }
    }
};

void say(char *msg, size_t cap, const char *fmt, ...) {
    if (!msg || !cap) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(msg, cap, fmt, ap);
    va_end(ap);
}

// getline with the buffer freed at scope exit.
struct LineReader {
    char *buf = nullptr;
    size_t cap = 0;
    ~LineReader() { free(buf); }
    bool next(FILE *f, std::string *line) {
        const ssize_t n = getline(&buf, &cap, f);
        if (n < 0) return false;
        line->assign(buf, static_cast<size_t>(n));
        return true;
    }
};

// Splits a record at tabs (the path of a FILE record is the rest of the line).
std::vector<std::string> fields(const std::string &line, size_t max_fields) {
    std::vector<std::string> out;
    size_t at = 0;
    while (out.size() + 1 < max_fields) {
        const size_t tab = line.find('\t', at);
        if (tab == std::string::npos) break;
        out.push_back(line.substr(at, tab - at));
        at = tab + 1;
    }
    out.push_back(line.substr(at));
    return out;
}

bool to_u64(const std::string &s, uint64_t *v) {
    if (s.empty() || s.size() > 20) return false;
    for (char c : s)
        if (c < '0' || c > '9') return false;
    errno = 0;
    char *end = nullptr;
    const unsigned long long x = strtoull(s.c_str(), &end, 10);
    if (errno || *end) return false;
    *v = x;
    return true;
}

bool to_int(const std::string &s, int *v) {
    uint64_t x = 0;
    if (s.size() > 1 && s[0] == '-') {
        if (!to_u64(s.substr(1), &x) || x > (uint64_t)INT_MAX) return false;
        *v = -static_cast<int>(x);
        return true;
    }
    if (!to_u64(s, &x) || x > (uint64_t)INT_MAX) return false;
    *v = static_cast<int>(x);
    return true;
}

int parse_index(FILE *f, WeightIndex *ix, char *msg, size_t cap) {
    LineReader lines;
    auto read_line = [&](std::string *line) { return lines.next(f, line); };
    std::string line;
    if (!read_line(&line) || line != "COB_QWEN_INDEX_V1\n") {
        say(msg, cap, "not a COB_QWEN_INDEX_V1 index");
        return cudaErrorInvalidValue;
    }
    if (!read_line(&line) || line != "VERIFIED 1\n") {
        say(msg, cap, "the index does not record verified weights (VERIFIED 1)");
        return cudaErrorInvalidValue;
    }
    // 35 whitespace-separated header numbers, possibly over several lines
    std::vector<std::string> words;
    while (words.size() < 36 && read_line(&line)) {
        size_t at = 0;
        while (at < line.size()) {
            while (at < line.size() && isspace(static_cast<unsigned char>(line[at]))) at++;
            size_t end = at;
            while (end < line.size() && !isspace(static_cast<unsigned char>(line[end]))) end++;
            if (end > at) words.push_back(line.substr(at, end - at));
            at = end;
        }
    }
    bool ok = words.size() == 36;
    for (int j = 0; ok && j < 3; j++) ok = to_u64(words[j], &ix->multipliers[j]);
    for (int j = 0; ok && j < 16; j++) ok = to_u64(words[3 + j], &ix->head_offsets[j]);
    for (int j = 0; ok && j < 16; j++) ok = to_u64(words[19 + j], &ix->head_vocab[j]) && ix->head_vocab[j] > 0;
    if (ok) ok = to_int(words[35], &ix->ple_eos);
    if (!ok) {
        say(msg, cap, "malformed index header numbers");
        return cudaErrorInvalidValue;
    }
    while (read_line(&line)) {
        if (line == "\n" || line == "\r\n") continue;
        while (!line.empty() && (line.back() == '\n' || line.back() == '\r')) line.pop_back();
        if (line.compare(0, 5, "FILE\t") == 0) {
            const std::vector<std::string> r = fields(line, 4);
            int id = -1;
            uint64_t bytes = 0;
            if (r.size() != 4 || !to_int(r[1], &id) || id < 0 || id >= kIndexFiles || !to_u64(r[2], &bytes) ||
                ix->files[id].fd >= 0 || r[3].empty()) {
                say(msg, cap, "malformed FILE record: %s", line.c_str());
                return cudaErrorInvalidValue;
            }
            MappedFile &mf = ix->files[id];
            mf.fd = open(r[3].c_str(), O_RDONLY);
            struct stat st;
            if (mf.fd < 0 || fstat(mf.fd, &st) || static_cast<uint64_t>(st.st_size) != bytes || bytes == 0) {
                say(msg, cap, "weights file missing or of the wrong size: %s", r[3].c_str());
                return cudaErrorFileNotFound;
            }
            void *p = mmap(nullptr, bytes, PROT_READ, MAP_PRIVATE, mf.fd, 0);
            if (p == MAP_FAILED) {
                say(msg, cap, "cannot map %s", r[3].c_str());
                return cudaErrorFileNotFound;
            }
            mf.data = static_cast<const unsigned char *>(p);
            mf.bytes = bytes;
        } else if (line.compare(0, 7, "TENSOR\t") == 0) {
            const std::vector<std::string> r = fields(line, 11);
            IndexTensor t;
            bool good = r.size() == 10 && !r[1].empty() && r[1].size() < 128 && to_int(r[2], &t.file) &&
                        to_u64(r[3], &t.offset) && to_u64(r[4], &t.bytes) && to_int(r[5], &t.type);
            for (int j = 0; good && j < 4; j++) good = to_u64(r[6 + j], &t.dims[j]);
            good = good && t.file >= 0 && t.file < kIndexFiles && ix->files[t.file].data && t.bytes > 0 &&
                   t.offset <= ix->files[t.file].bytes && t.bytes <= ix->files[t.file].bytes - t.offset &&
                   ix->tensors.size() < kIndexTensors && !ix->tensors.count(r[1]);
            uint64_t expect = 0;
            good = good && qg_tensor_bytes(t.type, t.dims, &expect) == 0 && expect == t.bytes;
            if (!good) {
                say(msg, cap, "malformed or unsupported TENSOR record: %s", line.c_str());
                return cudaErrorInvalidValue;
            }
            ix->tensors.emplace(r[1], t);
        } else {
            say(msg, cap, "unexpected index line: %s", line.c_str());
            return cudaErrorInvalidValue;
        }
    }
    return cudaSuccess;
}

}  // namespace

extern "C" int qg_index_open(const char *path, void **index, char *message, size_t message_bytes) {
    if (message && message_bytes) message[0] = 0;
    if (!path || !index) return cudaErrorInvalidValue;
    *index = nullptr;
    FILE *f = fopen(path, "r");
    if (!f) {
        say(message, message_bytes, "cannot open the index %s", path);
        return cudaErrorFileNotFound;
    }
    auto *ix = new (std::nothrow) WeightIndex;
    if (!ix) {
        fclose(f);
        return cudaErrorMemoryAllocation;
    }
    const int rc = parse_index(f, ix, message, message_bytes);
    fclose(f);
    if (rc) {
        delete ix;
        return rc;
    }
    *index = ix;
    return cudaSuccess;
}

extern "C" void qg_index_close(void *index) { delete static_cast<WeightIndex *>(index); }

extern "C" int qg_index_tensor(const void *index, const char *name, const void **host, int *type, uint64_t dims[4],
                               uint64_t *bytes) {
    const auto *ix = static_cast<const WeightIndex *>(index);
    if (!ix || !name) return cudaErrorInvalidValue;
    const auto it = ix->tensors.find(name);
    if (it == ix->tensors.end()) return cudaErrorInvalidValue;
    const IndexTensor &t = it->second;
    if (host) *host = ix->files[t.file].data + t.offset;
    if (type) *type = t.type;
    if (dims) memcpy(dims, t.dims, sizeof(t.dims));
    if (bytes) *bytes = t.bytes;
    return cudaSuccess;
}

// ---------------------------------------------------------------- route traces
namespace {
struct RouteTrace {
    FILE *f = nullptr;
    ~RouteTrace() {
        if (f) fclose(f);
    }
};
}  // namespace

extern "C" int qg_route_trace_open(const char *path, void **trace) {
    if (!path || !trace) return cudaErrorInvalidValue;
    *trace = nullptr;
    auto *t = new (std::nothrow) RouteTrace;
    if (!t) return cudaErrorMemoryAllocation;
    t->f = fopen(path, "rb");
    char magic[8];
    if (!t->f) {
        delete t;
        return cudaErrorFileNotFound;
    }
    if (fread(magic, 1, 8, t->f) != 8 || memcmp(magic, "QROUTE1\n", 8) != 0) {
        delete t;
        return cudaErrorInvalidValue;
    }
    *trace = t;
    return cudaSuccess;
}

extern "C" int qg_route_trace_next(void *trace, int *layer, int *position, int *tokens, int *ids, float *weights,
                                   int capacity) {
    auto *t = static_cast<RouteTrace *>(trace);
    if (!t || !layer || !position || !tokens || !ids || !weights || capacity < 1) return cudaErrorInvalidValue;
    uint32_t head[3];
    const size_t got = fread(head, sizeof(uint32_t), 3, t->f);
    if (got == 0 && feof(t->f)) {  // clean end: no more records
        *tokens = 0;
        return cudaSuccess;
    }
    if (got != 3 || head[2] < 1 || head[2] > static_cast<uint32_t>(nb::kMaxTokens) ||
        head[2] > static_cast<uint32_t>(capacity) || head[0] > static_cast<uint32_t>(INT_MAX) ||
        head[1] > static_cast<uint32_t>(INT_MAX))
        return cudaErrorInvalidValue;
    const size_t n = static_cast<size_t>(head[2]) * nb::kTop;
    if (fread(ids, sizeof(int), n, t->f) != n || fread(weights, sizeof(float), n, t->f) != n)
        return cudaErrorInvalidValue;  // truncated record
    *layer = static_cast<int>(head[0]);
    *position = static_cast<int>(head[1]);
    *tokens = static_cast<int>(head[2]);
    return cudaSuccess;
}

extern "C" void qg_route_trace_close(void *trace) { delete static_cast<RouteTrace *>(trace); }
