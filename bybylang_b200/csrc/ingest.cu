// ingest.cu - weight ingestion: read-only checkpoint mappings (mapped_file.nim), the copy
// engine that moves a mapped or otherwise pageable host range into HBM (the dGPU branch of
// residentUploadQ4Mapped / sessionUploadPrivatePtr, gpubackend.nim:2920-2998), the sampled
// content fingerprint (probe_data.nim:4-33) and the checkpoint tensor index of NIMQ2, NIMQ3,
// NIMBIN and safetensors files (probeTensorIndex, probe_weights.nim:29-104).
//
// A B200 sits behind a PCIe / C2C link, not on the host's memory: weights are copied into HBM
// once, at load.  A pageable range (a file mapping) cannot be the source of an asynchronous
// DMA, so the driver would stage it through a small pinned buffer of its own, one piece at a
// time.  The engine here stages it instead through pinned slots of its own, several host
// threads at once: each thread touches (page-faults in) and copies its share of the range into
// its slots while the copy engine drains the previous slots, so file reads, memcpy and DMA
// overlap.  BYBY_CUDA_INGEST=register pins the range itself in place (cudaHostRegister,
// read-only) and copies it with one DMA, falling back to staging where the range cannot be
// pinned.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "json.cuh"
#include "kernels.h"

namespace bybycu {
namespace ingest {

constexpr size_t kSlotBytes = size_t(8) << 20;   // one staging slot
constexpr int kSlots = 2;                         // per worker: one filling, one draining
constexpr int kMaxWorkers = 16;
constexpr size_t kDirectBytes = size_t(4) << 20;  // below this, one plain copy

struct Worker {
    cudaStream_t st = nullptr;
    void* slot[kSlots] = {};
    cudaEvent_t ev[kSlots] = {};
};

// Per device: the workers' streams and pinned slots, made on first use and kept.  One staged
// upload runs at a time per device.
struct Engine {
    std::mutex mu;
    std::vector<Worker> workers;
};
std::mutex g_engines_mu;
std::map<int, Engine*> g_engines;

// One worker per host thread, up to 16 (on a 16-thread host, 2 GiB from a warm page cache:
// 1 worker 11.8 GB/s, 4: 31, 8: 36, 16: 48 - the pinned-DMA rate of the link).
int workers_wanted() {
    int n = kMaxWorkers;
    if (const char* e = getenv("BYBY_CUDA_INGEST_THREADS")) n = atoi(e);
    const int hw = static_cast<int>(std::thread::hardware_concurrency());
    if (hw > 0) n = std::min(n, hw);
    return std::max(1, std::min(n, kMaxWorkers));
}

Engine* engine(int device) {
    std::lock_guard<std::mutex> lock(g_engines_mu);
    auto it = g_engines.find(device);
    if (it == g_engines.end()) it = g_engines.emplace(device, new Engine).first;
    return it->second;
}

// Grows the engine to n workers (the caller holds eng->mu).
int ensure_workers(Engine* eng, int n) {
    while (static_cast<int>(eng->workers.size()) < n) {
        Worker w;
        BYBYCU_CUDA_TRY(cudaStreamCreateWithFlags(&w.st, cudaStreamNonBlocking));
        for (int s = 0; s < kSlots; ++s) {
            BYBYCU_CUDA_TRY(cudaHostAlloc(&w.slot[s], kSlotBytes, cudaHostAllocPortable));
            BYBYCU_CUDA_TRY(cudaEventCreateWithFlags(&w.ev[s], cudaEventDisableTiming));
        }
        eng->workers.push_back(w);
    }
    return BYBYCU_OK;
}

// Chunk c of the range goes to worker c % n, slot (c / n) % 2.  Each worker waits for its
// slot's previous copy before refilling it.
int staged_upload(uint8_t* dst, const uint8_t* src, size_t bytes, int device) {
    const int n = workers_wanted();
    Engine* eng = engine(device);
    std::lock_guard<std::mutex> lock(eng->mu);
    if (int rc = ensure_workers(eng, n)) return rc;
    const size_t n_chunks = (bytes + kSlotBytes - 1) / kSlotBytes;
    const int used = static_cast<int>(std::min<size_t>(n, n_chunks));
    std::atomic<int> first_err{0};
    std::vector<cudaError_t> errs(used, cudaSuccess);
    auto work = [&](int w) {
        Worker& wk = eng->workers[w];
        cudaError_t e = cudaSetDevice(device);
        bool pending[kSlots] = {};
        for (size_t c = w, i = 0; c < n_chunks && e == cudaSuccess && !first_err.load(std::memory_order_relaxed);
             c += used, ++i) {
            const int s = static_cast<int>(i % kSlots);
            if (pending[s]) e = cudaEventSynchronize(wk.ev[s]);
            if (e != cudaSuccess) break;
            const size_t off = c * kSlotBytes, len = std::min(kSlotBytes, bytes - off);
            memcpy(wk.slot[s], src + off, len);
            e = cudaMemcpyAsync(dst + off, wk.slot[s], len, cudaMemcpyHostToDevice, wk.st);
            if (e == cudaSuccess) e = cudaEventRecord(wk.ev[s], wk.st);
            pending[s] = true;
        }
        const cudaError_t e2 = cudaStreamSynchronize(wk.st);
        if (e == cudaSuccess) e = e2;
        errs[w] = e;
        if (e != cudaSuccess) first_err.store(1, std::memory_order_relaxed);
    };
    std::vector<std::thread> threads;
    threads.reserve(used > 0 ? used - 1 : 0);
    for (int w = 1; w < used; ++w) threads.emplace_back(work, w);
    work(0);
    for (auto& t : threads) t.join();
    for (cudaError_t e : errs)
        if (e != cudaSuccess) return cuda_fail(e, "staged host-to-device copy");
    return BYBYCU_OK;
}

// Pins the pages of [src, src + bytes) in place and copies them with one DMA.  Returns
// false (nothing done) when the range cannot be pinned.
bool registered_upload(uint8_t* dst, const uint8_t* src, size_t bytes, int* rc) {
    const uintptr_t page = static_cast<uintptr_t>(sysconf(_SC_PAGESIZE));
    const uintptr_t b = reinterpret_cast<uintptr_t>(src) & ~(page - 1);
    const uintptr_t e = (reinterpret_cast<uintptr_t>(src) + bytes + page - 1) & ~(page - 1);
    void* base = reinterpret_cast<void*>(b);
    if (cudaHostRegister(base, e - b, cudaHostRegisterReadOnly | cudaHostRegisterPortable) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    cudaError_t err = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
    const cudaError_t err2 = cudaHostUnregister(base);
    if (err == cudaSuccess) err = err2;
    *rc = err == cudaSuccess ? BYBYCU_OK : cuda_fail(err, "registered host-to-device copy");
    return true;
}

bool use_register() {
    const char* e = getenv("BYBY_CUDA_INGEST");
    return e && !strcmp(e, "register");
}

// ---------------------------------------------------------------------------------------
// Fingerprint (probe_data.nim:4-17): FNV-1a over the byte count and 5 sampled 64-byte runs
// ---------------------------------------------------------------------------------------
std::vector<int64_t> fingerprint_offsets(int64_t bytes) {
    std::vector<int64_t> r;
    if (bytes <= 0) return r;
    const int64_t width = std::min<int64_t>(64, bytes);
    for (int i = 0; i <= 4; ++i) {
        const int64_t off = (bytes - width) * i / 4;
        if (std::find(r.begin(), r.end(), off) == r.end()) r.push_back(off);
    }
    return r;
}

template <class Read>
void fingerprint_text(int64_t bytes, Read read_at, char* out, int out_len) {
    uint64_t h = 0xcbf29ce484222325ull;
    for (int i = 0; i < 8; ++i) h = (h ^ ((static_cast<uint64_t>(bytes) >> (8 * i)) & 255u)) * 0x100000001b3ull;
    const int64_t width = std::min<int64_t>(64, bytes);
    uint8_t blk[64];
    for (int64_t off : fingerprint_offsets(bytes)) {
        read_at(off, blk, width);
        for (int64_t j = 0; j < width; ++j) h = (h ^ blk[j]) * 0x100000001b3ull;
    }
    snprintf(out, static_cast<size_t>(out_len), "sample1-%016llx", static_cast<unsigned long long>(h));
}

// ---------------------------------------------------------------------------------------
// Checkpoint index (probe_weights.nim:29-104)
// ---------------------------------------------------------------------------------------
struct Reader {
    FILE* f = nullptr;
    int64_t size = 0;
    bool ok = true;
    std::string err;
    void fail(const char* m) {
        if (ok) err = m;
        ok = false;
    }
    bool read(void* p, size_t n) {
        if (!ok) return false;
        if (fread(p, 1, n, f) != n) return false;
        return true;
    }
    int64_t pos() { return ok ? static_cast<int64_t>(ftello(f)) : 0; }
    void seek(int64_t p) {
        if (ok && fseeko(f, static_cast<off_t>(p), SEEK_SET) != 0) fail("checkpoint seek failed");
    }
    int32_t i32() {
        int32_t v = 0;
        if (!read(&v, 4)) fail("truncated checkpoint header");
        return v;
    }
    int64_t i64_count() {
        int64_t v = 0;
        if (!read(&v, 8)) fail("truncated checkpoint header");
        else if (v < 0) fail("invalid checkpoint element count");
        return v;
    }
    std::string string() {
        const int32_t n = i32();
        std::string s;
        if (!ok) return s;
        if (n < 0 || n > (1 << 24)) {
            fail("invalid checkpoint string length");
            return s;
        }
        s.resize(static_cast<size_t>(n));
        if (n > 0 && !read(&s[0], static_cast<size_t>(n))) fail("truncated checkpoint string");
        return s;
    }
};

void set_name(bybycu_tensor_info* t, const std::string& name) {
    snprintf(t->name, sizeof t->name, "%s", name.c_str());
    t->name_len = static_cast<int32_t>(std::min<size_t>(name.size(), INT32_MAX));
}

bool ends_with(const std::string& s, const char* suf) {
    const size_t n = strlen(suf);
    return s.size() >= n && !s.compare(s.size() - n, n, suf);
}

int index_file(const char* path, std::vector<bybycu_tensor_info>* out, std::string* err) {
    Reader r;
    r.f = fopen(path, "rb");
    if (!r.f) {
        *err = std::string("cannot open checkpoint: ") + path;
        return BYBYCU_ERR_ARGS;
    }
    struct stat st;
    if (fstat(fileno(r.f), &st) != 0) {
        fclose(r.f);
        *err = "cannot stat checkpoint";
        return BYBYCU_ERR_ARGS;
    }
    r.size = static_cast<int64_t>(st.st_size);
    const std::string p(path);
    if (ends_with(p, ".safetensors")) {
        uint64_t header_bytes = 0;
        if (!r.read(&header_bytes, 8) || header_bytes > (uint64_t(1) << 28)) r.fail("invalid safetensors header");
        std::string text;
        if (r.ok) {
            text.resize(static_cast<size_t>(header_bytes));
            if (header_bytes && !r.read(&text[0], text.size())) r.fail("truncated safetensors header");
        }
        JVal h;
        if (r.ok && (!json_parse(text, &h) || h.type != JVal::kObj)) r.fail("invalid safetensors header");
        for (size_t i = 0; r.ok && i < h.obj.size(); ++i) {
            const auto& kv = h.obj[i];
            if (kv.first == "__metadata__") continue;
            const JVal* dt = kv.second.get("dtype");
            const JVal* sh = kv.second.get("shape");
            const JVal* of = kv.second.get("data_offsets");
            if (!dt || dt->type != JVal::kStr || !sh || sh->type != JVal::kArr || !of || of->type != JVal::kArr ||
                of->arr.size() != 2 || of->arr[0].type != JVal::kNum || of->arr[1].type != JVal::kNum ||
                sh->arr.size() > 8) {
                r.fail("invalid safetensors header");
                break;
            }
            bybycu_tensor_info t{};
            set_name(&t, kv.first);
            t.kind = dt->str == "F32" ? 0 : -1;
            snprintf(t.dtype, sizeof t.dtype, "%s", dt->str.c_str());
            t.offset = 8 + static_cast<int64_t>(header_bytes) + static_cast<int64_t>(of->arr[0].num);
            t.bytes = static_cast<int64_t>(of->arr[1].num) - static_cast<int64_t>(of->arr[0].num);
            t.rank = static_cast<int32_t>(sh->arr.size());
            for (size_t d = 0; d < sh->arr.size(); ++d) {
                if (sh->arr[d].type != JVal::kNum) { r.fail("invalid safetensors header"); break; }
                t.shape[d] = static_cast<int64_t>(sh->arr[d].num);
            }
            out->push_back(t);
        }
    } else {
        char prefix[8] = {0};
        if (!r.read(prefix, 8)) r.fail("truncated checkpoint header");
        r.seek(0);
        if (r.ok && !memcmp(prefix, "NIMBIN", 6)) {   // raw fp32 state dict
            r.seek(8);
            const int32_t meta = r.i32();
            if (r.ok && (meta < 0 || meta > 1000000)) r.fail("invalid .bin metadata");
            for (int32_t i = 0; r.ok && i < meta; ++i) {
                r.string();
                r.string();
            }
            const int32_t count = r.i32();
            if (r.ok && (count < 0 || count > 1000000)) r.fail("invalid tensor count");
            for (int32_t i = 0; r.ok && i < count; ++i) {
                bybycu_tensor_info t{};
                set_name(&t, r.string());
                t.kind = 0;
                const int32_t rank = r.i32();
                if (r.ok && (rank < 0 || rank > 8)) r.fail("invalid tensor rank");
                t.rank = rank;
                for (int32_t d = 0; r.ok && d < rank; ++d) t.shape[d] = r.i32();
                const int64_t elems = r.i64_count();
                if (r.ok && elems > r.size / 4) r.fail("invalid .bin tensor element count");
                t.bytes = elems * 4;
                t.offset = r.pos();
                r.seek(t.offset + t.bytes);
                if (r.ok) out->push_back(t);
            }
        } else if (r.ok) {
            const std::string magic = r.string();
            int32_t alignment = 0;
            if (r.ok && magic == "NIMQ3") {
                alignment = r.i32();
                if (r.ok && (alignment < 64 || alignment > (1 << 24))) r.fail("invalid NIMQ3 alignment");
                r.seek(alignment);
            } else if (r.ok && magic != "NIMQ2") {
                *err = "unsupported checkpoint format: " + magic;
                fclose(r.f);
                return BYBYCU_ERR_ARGS;
            }
            for (int i = 0; i < 5; ++i) r.i32();
            const int32_t count = r.i32();
            if (r.ok && (count < 0 || count > 1000000)) r.fail("invalid tensor count");
            for (int32_t i = 0; r.ok && i < count; ++i) {
                bybycu_tensor_info t{};
                set_name(&t, r.string());
                uint8_t kind = 0;
                if (r.ok && !r.read(&kind, 1)) r.fail("truncated tensor kind");
                t.kind = kind;
                const int32_t rank = r.i32();
                if (r.ok && (rank < 0 || rank > 8)) r.fail("invalid tensor rank");
                t.rank = rank;
                for (int32_t d = 0; r.ok && d < rank; ++d) t.shape[d] = r.i32();
                t.scales = r.i32();
                if (r.ok && t.scales < 0) r.fail("invalid tensor scale count");
                t.scale_offset = r.pos();
                r.seek(t.scale_offset + static_cast<int64_t>(t.scales) * 8);
                t.group_size = r.i32();
                t.eb = r.i32();
                t.mb = r.i32();
                t.bytes = r.i32();
                if (r.ok && t.bytes < 0) {
                    fclose(r.f);
                    *err = std::string("checkpoint tensor outside file: ") + t.name;
                    return BYBYCU_ERR_RANGE;
                }
                if (alignment > 0) {
                    const int64_t at = r.pos();
                    r.seek(at + (alignment - at % alignment) % alignment);
                }
                t.offset = r.pos();
                r.seek(t.offset + t.bytes);
                if (r.ok) out->push_back(t);
            }
        }
    }
    fclose(r.f);
    if (!r.ok) {
        *err = r.err;
        return BYBYCU_ERR_ARGS;
    }
    for (const auto& t : *out)
        if (t.offset < 0 || t.bytes < 0 || t.offset + t.bytes > r.size) {
            *err = std::string("checkpoint tensor outside file: ") + t.name;
            return BYBYCU_ERR_RANGE;
        }
    return BYBYCU_OK;
}

struct Mapping {
    void* data = nullptr;
    size_t size = 0;
};

}  // namespace ingest

int upload_host_range(void* dst, const void* src, int64_t bytes) {
    using namespace ingest;
    if (bytes <= 0) return BYBYCU_OK;
    const size_t n = static_cast<size_t>(bytes);
    if (n < kDirectBytes) {
        BYBYCU_CUDA_TRY(cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice));
        return BYBYCU_OK;
    }
    int device = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&device));
    // page-locked memory needs no staging
    cudaPointerAttributes pa;
    if (cudaPointerGetAttributes(&pa, src) == cudaSuccess && pa.type == cudaMemoryTypeHost) {
        BYBYCU_CUDA_TRY(cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice));
        return BYBYCU_OK;
    }
    cudaGetLastError();
    int rc = BYBYCU_OK;
    if (use_register() && registered_upload(static_cast<uint8_t*>(dst), static_cast<const uint8_t*>(src), n, &rc))
        return rc;
    return staged_upload(static_cast<uint8_t*>(dst), static_cast<const uint8_t*>(src), n, device);
}

}  // namespace bybycu

using namespace bybycu;

extern "C" {

int bybycu_map_file(const char* path, void** data, int64_t* size, void** mapping) {
    if (!path || !data || !size || !mapping) return set_error(BYBYCU_ERR_ARGS, "map_file: NULL argument");
    *data = nullptr;
    *size = 0;
    *mapping = nullptr;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return set_error(BYBYCU_ERR_ARGS, "cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size <= 0) {
        close(fd);
        return set_error(BYBYCU_ERR_ARGS, "cannot map %s: empty or unreadable", path);
    }
    void* p = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return set_error(BYBYCU_ERR_ARGS, "cannot map %s", path);
    madvise(p, static_cast<size_t>(st.st_size), MADV_SEQUENTIAL);
    auto* m = new ingest::Mapping;
    m->data = p;
    m->size = static_cast<size_t>(st.st_size);
    *data = p;
    *size = static_cast<int64_t>(st.st_size);
    *mapping = m;
    return BYBYCU_OK;
}

int bybycu_unmap_file(void* mapping) {
    if (!mapping) return BYBYCU_OK;
    auto* m = static_cast<ingest::Mapping*>(mapping);
    if (m->data) munmap(m->data, m->size);
    delete m;
    return BYBYCU_OK;
}

int bybycu_upload_host_range(void* dst, const void* src, int64_t bytes) {
    if (bytes < 0 || (bytes > 0 && (!dst || !src))) return set_error(BYBYCU_ERR_ARGS, "upload_host_range: bad arguments");
    return upload_host_range(dst, src, bytes);
}

int bybycu_fingerprint(const void* data, int64_t bytes, char* out, int out_len) {
    if (!out || out_len < 25 || bytes < 0 || (bytes > 0 && !data))
        return set_error(BYBYCU_ERR_ARGS, "fingerprint: bad arguments");
    const uint8_t* p = static_cast<const uint8_t*>(data);
    ingest::fingerprint_text(bytes, [&](int64_t off, uint8_t* dst, int64_t n) { memcpy(dst, p + off, n); }, out,
                             out_len);
    return BYBYCU_OK;
}

int bybycu_checkpoint_index(const char* path, bybycu_tensor_info* out, int cap, int* count) {
    if (!path || !count || cap < 0 || (cap > 0 && !out)) return set_error(BYBYCU_ERR_ARGS, "checkpoint_index: bad arguments");
    *count = 0;
    std::vector<bybycu_tensor_info> idx;
    std::string err;
    if (int rc = ingest::index_file(path, &idx, &err)) return set_error(rc, "%s", err.c_str());
    *count = static_cast<int>(idx.size());
    for (int i = 0; i < cap && i < static_cast<int>(idx.size()); ++i) out[i] = idx[i];
    return BYBYCU_OK;
}

}  // extern "C"
