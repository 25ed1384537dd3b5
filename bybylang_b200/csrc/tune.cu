// tune.cu - tuned launch plans: the CUDA side of the reference's Q4 autotuner
// (vulkanPrepareQ4Tuned, backends/vulkan/q4_autotune.nim:387-543) and of its plan cache
// (q4_autotune.nim:32-117).
//
// A plan is a route (SIMT, GEMV, TC) and that route's launch knobs (the operand form of the
// M = 1 GEMV, the ring depth of its weight stream, CTAs per SM of the fp16 GEMV).  Preparing a
// shape runs every candidate the device supports on the caller's weights and a fixed input,
// keeps those whose output matches the reference candidate's (the bit-exact route, run first)
// within the tolerance of their arithmetic, times the survivors and installs the fastest in a
// per-process table that the automatic route consults.  As in the reference:
//   * candidate 0 is the reference kernel; it must run and give finite values, or nothing is
//     prepared;
//   * parity: max |v - ref| <= max(1e-5, max |ref| * tol), tol = 3e-3, the reference's bound
//     for candidates with narrow (fp16 / bf16 / integer) operands, which every candidate here
//     has besides the reference itself (q4_autotune.nim:485-505);
//   * timing: three rounds, the order reversed every other round, the median kept; a
//     candidate replaces the current best only when it is 3% faster (q4_autotune.nim:506-532);
//   * the input is x[i] = ((17 i) mod 101 - 50) / 64 (q4_autotune.nim:462-463);
//   * the decode shape (M = 1) and the prefill shapes have separate plans; prefill shapes are
//     tuned at a representative M.  Where the reference keeps one prefill plan (tuned at
//     M = 64), plans here are per power-of-two class of M (2, 4, ..., 128; above 128 the 128
//     plan), since the best route changes between a few rows and a full tile;
//   * chosen plans persist in a JSON file named for a hash of the device, driver, library
//     build and route switches, in <cache dir>/q4-plans-<hash>.json, written atomically.
//
// B200-specific measurement: candidates are timed on a private stream behind a short,
// self-ending hold kernel, so that the host enqueues the whole batch before the first
// launch runs and the events bracket back-to-back device time (the GEMVs take a few
// microseconds, about as long as enqueuing one).  The batch cycles over copies of the
// weights that together exceed the 126 MB L2, as consecutive layers of a decode step do.
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "json.cuh"
#include "kernels.h"

#ifndef BYBYCU_SOURCE_HASH
#define BYBYCU_SOURCE_HASH 0u
#endif

namespace bybycu {

int tile_gemm_impl(int fmt, int M, int K, int N, const void* x, int x_dtype, int64_t x_len, const void* packed,
                   int64_t packed_len, int64_t scale_base, const float* lut, int64_t lut_len, int64_t lut_base,
                   void* out, int out_dtype, int64_t out_len, int route, cudaStream_t stream);
int check_tile_gemm(int fmt, int M, int K, int N, int64_t x_len, int64_t packed_len, int64_t scale_base,
                    int64_t lut_len, int64_t lut_base, int64_t out_len);

namespace tune {

constexpr int kCacheVersion = 1;
constexpr int kMaxClass = 128;                       // prefill classes 2, 4, ..., 128
constexpr float kTolNarrow = 3e-3f;
constexpr size_t kColdBytes = size_t(256) << 20;     // weight copies cycled while timing (> L2)
constexpr int kMaxCopies = 16;

// A plan's shape: the op, the tile format and activation type (tile GEMM), the group layout
// (matmul_q4), K, N and the class of M, on one device.
struct Key {
    int device, op, fmt, xdt, K, N, group, groups, mclass;
    bool operator<(const Key& o) const {
        return std::tie(device, op, fmt, xdt, K, N, group, groups, mclass) <
               std::tie(o.device, o.op, o.fmt, o.xdt, o.K, o.N, o.group, o.groups, o.mclass);
    }
};

std::mutex g_mu;
std::map<Key, bybycu_plan> g_plans;
std::atomic<int> g_count{0};
std::atomic<long long> g_dispatches{0};

int mclass_of(int M) {
    if (M <= 1) return 1;
    int c = 2;
    while (c < M && c < kMaxClass) c <<= 1;
    return c;
}

bool find_plan(const Key& k, bybycu_plan* out) {
    if (g_count.load(std::memory_order_acquire) == 0) return false;
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_plans.find(k);
    if (it == g_plans.end()) return false;
    *out = it->second;
    return true;
}

void install(const Key& k, const bybycu_plan& p) {
    std::lock_guard<std::mutex> lock(g_mu);
    g_plans[k] = p;
    g_count.store(static_cast<int>(g_plans.size()), std::memory_order_release);
}

bool env_off(const char* name) {
    const char* e = getenv(name);
    return e && !strcmp(e, "0");
}

bool verbose() {
    const char* e = getenv("BYBY_Q4_TUNE_VERBOSE");
    return e && !strcmp(e, "1");
}

std::string key_string(const Key& k) {
    char b[160];
    snprintf(b, sizeof b, "op=%d;fmt=%d;x=%d;K=%d;N=%d;group=%d;groups=%d;M=%d", k.op, k.fmt, k.xdt, k.K, k.N, k.group,
             k.groups, k.mclass);
    return b;
}

// ---------------------------------------------------------------------------------------
// The plan cache file
// ---------------------------------------------------------------------------------------

// Stable FNV-1a (the reference's q4StableHash, q4_autotune.nim:26-30): an on-disk key must
// not change between processes.
uint64_t fnv1a(const std::string& s) {
    uint64_t h = 14695981039346656037ull;
    for (unsigned char c : s) h = (h ^ c) * 1099511628211ull;
    return h;
}

// Everything that changes which candidate wins or whether its output is right: the device,
// the driver and runtime, this library's ABI and sources, and the route switches read from
// the environment (q4TuneCacheSignature, q4_autotune.nim:37-60).
int signature(int device, std::string* out) {
    cudaDeviceProp prop;
    BYBYCU_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
    int drv = 0, rt = 0;
    BYBYCU_CUDA_TRY(cudaDriverGetVersion(&drv));
    BYBYCU_CUDA_TRY(cudaRuntimeGetVersion(&rt));
    const char* m1 = getenv("BYBY_CUDA_GEMV_M1");
    const char* st = getenv("BYBY_CUDA_GEMV_STAGES");
    char b[512];
    snprintf(b, sizeof b,
             "version=%d;device=%s;cc=%d.%d;sms=%d;l2=%d;mem_clock=%d;bus=%d;driver=%d;runtime=%d;abi=%d;"
             "source=%08x;gemv_m1=%s;gemv_stages=%s",
             kCacheVersion, prop.name, prop.major, prop.minor, prop.multiProcessorCount, prop.l2CacheSize,
             prop.memoryClockRate, prop.memoryBusWidth, drv, rt, BYBYCU_ABI_VERSION,
             static_cast<unsigned>(BYBYCU_SOURCE_HASH), m1 ? m1 : "", st ? st : "");
    *out = b;
    return BYBYCU_OK;
}

// BYBY_CUDA_TUNE_DIR, else $XDG_CACHE_HOME/bybylang_b200, else ~/.cache/bybylang_b200;
// BYBY_CUDA_TUNE_DIR=0 keeps plans in memory only.
std::string cache_dir() {
    if (const char* e = getenv("BYBY_CUDA_TUNE_DIR")) return strcmp(e, "0") ? std::string(e) : std::string();
    if (const char* x = getenv("XDG_CACHE_HOME"); x && *x) return std::string(x) + "/bybylang_b200";
    if (const char* h = getenv("HOME"); h && *h) return std::string(h) + "/.cache/bybylang_b200";
    return std::string();
}

int cache_path(int device, std::string* path) {
    path->clear();
    const std::string dir = cache_dir();
    if (dir.empty()) return BYBYCU_OK;
    std::string sig;
    if (int rc = signature(device, &sig)) return rc;
    char b[32];
    snprintf(b, sizeof b, "/q4-plans-%016llx.json", static_cast<unsigned long long>(fnv1a(sig)));
    *path = dir + b;
    return BYBYCU_OK;
}

std::string json_escape(const std::string& s) {
    std::string o;
    for (char c : s) {
        if (c == '"' || c == '\\') { o.push_back('\\'); o.push_back(c); }
        else if (static_cast<unsigned char>(c) < 0x20) o.push_back(' ');
        else o.push_back(c);
    }
    return o;
}

// The cached plans of one file, read once per process (q4LoadTuneCache).
std::mutex g_cache_mu;
std::map<std::string, std::map<std::string, bybycu_plan>> g_cache;   // path -> key -> plan

std::map<std::string, bybycu_plan>& cache_for(const std::string& path, const std::string& sig) {
    auto it = g_cache.find(path);
    if (it != g_cache.end()) return it->second;
    auto& plans = g_cache[path];
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return plans;
    std::string text;
    char buf[4096];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0 && text.size() < (size_t(8) << 20)) text.append(buf, n);
    fclose(f);
    JVal root;
    if (!json_parse(text, &root) || root.type != JVal::kObj) return plans;
    const JVal* ver = root.get("version");
    const JVal* s = root.get("signature");
    const JVal* ps = root.get("plans");
    if (!ver || ver->type != JVal::kNum || static_cast<int>(ver->num) != kCacheVersion || !s || s->str != sig || !ps ||
        ps->type != JVal::kObj)
        return plans;
    for (const auto& kv : ps->obj) {
        const JVal& e = kv.second;
        const JVal *r = e.get("route"), *va = e.get("variant"), *sg = e.get("stages"), *ms = e.get("ms"),
                   *nm = e.get("name");
        if (!r || !va || !sg || r->type != JVal::kNum || va->type != JVal::kNum || sg->type != JVal::kNum) continue;
        bybycu_plan p{};
        p.route = static_cast<int32_t>(r->num);
        p.variant = static_cast<int32_t>(va->num);
        p.stages = static_cast<int32_t>(sg->num);
        p.ms = ms && ms->type == JVal::kNum ? static_cast<float>(ms->num) : 0.0f;
        if (nm && nm->type == JVal::kStr) snprintf(p.name, sizeof p.name, "%s", nm->str.c_str());
        if (p.route != BYBYCU_ROUTE_SIMT && p.route != BYBYCU_ROUTE_GEMV && p.route != BYBYCU_ROUTE_TC) continue;
        plans[kv.first] = p;
    }
    return plans;
}

bool cached_plan(int device, const Key& k, bybycu_plan* out) {
    std::string path, sig;
    if (cache_path(device, &path) || path.empty() || signature(device, &sig)) {
        cudaGetLastError();
        return false;
    }
    std::lock_guard<std::mutex> lock(g_cache_mu);
    auto& plans = cache_for(path, sig);
    auto it = plans.find(key_string(k));
    if (it == plans.end()) return false;
    *out = it->second;
    return true;
}

void mkdirs(const std::string& dir) {
    for (size_t i = 1; i <= dir.size(); ++i)
        if (i == dir.size() || dir[i] == '/') mkdir(dir.substr(0, i).c_str(), 0755);
}

// q4SaveTuneCache: the file is rewritten whole through a temporary and a rename, so a reader
// never sees half of it.  A cache that cannot be written only costs the next process a tune.
void save_plan(int device, const Key& k, const bybycu_plan& p) {
    std::string path, sig;
    if (cache_path(device, &path) || path.empty() || signature(device, &sig)) {
        cudaGetLastError();
        return;
    }
    std::lock_guard<std::mutex> lock(g_cache_mu);
    auto& plans = cache_for(path, sig);
    plans[key_string(k)] = p;
    mkdirs(path.substr(0, path.rfind('/')));
    char tmp_suffix[32];
    snprintf(tmp_suffix, sizeof tmp_suffix, ".tmp.%d", static_cast<int>(getpid()));
    const std::string tmp = path + tmp_suffix;
    FILE* f = fopen(tmp.c_str(), "wb");
    if (!f) return;
    fprintf(f, "{\n  \"version\": %d,\n  \"signature\": \"%s\",\n  \"plans\": {", kCacheVersion, json_escape(sig).c_str());
    bool first = true;
    for (const auto& kv : plans) {
        const bybycu_plan& q = kv.second;
        fprintf(f, "%s\n    \"%s\": {\"name\": \"%s\", \"route\": %d, \"variant\": %d, \"stages\": %d, \"ms\": %.6g}",
                first ? "" : ",", json_escape(kv.first).c_str(), json_escape(q.name).c_str(), q.route, q.variant,
                q.stages, static_cast<double>(q.ms));
        first = false;
    }
    fprintf(f, "\n  }\n}\n");
    const bool ok = fflush(f) == 0;
    fclose(f);
    if (!ok || rename(tmp.c_str(), path.c_str()) != 0) unlink(tmp.c_str());
}

// ---------------------------------------------------------------------------------------
// Candidates, parity and timing
// ---------------------------------------------------------------------------------------

// Occupies the tuning stream for `ns` nanoseconds (it ends by itself) so that the launches
// queued behind it start back to back.
__global__ void tune_hold_kernel(uint64_t ns) {
    if (threadIdx.x != 0) return;
    const uint64_t t0 = globaltimer_ns();
    for (int i = 0; i < (1 << 22); ++i)
        if (globaltimer_ns() - t0 >= ns) break;
}

// x[i] = ((17 i) mod 101 - 50) / 64: exact in fp32 and in bf16.
__global__ void tune_input_kernel(void* x, int64_t n, int bf16) {
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const float v = static_cast<float>(static_cast<int>((i * 17) % 101) - 50) / 64.0f;
        if (bf16) static_cast<__nv_bfloat16*>(x)[i] = __float2bfloat16_rn(v);
        else static_cast<float*>(x)[i] = v;
    }
}

struct Cand {
    bybycu_plan plan;
    float tol;
};

// Runs plan `p` on weight copy `copy` into `out` on `st`.
using Runner = std::function<int(const bybycu_plan& p, int copy, float* out, cudaStream_t st)>;

bybycu_plan make_plan(int route, int variant, int stages, const char* fmt, ...) __attribute__((format(printf, 4, 5)));
bybycu_plan make_plan(int route, int variant, int stages, const char* fmt, ...) {
    bybycu_plan p{};
    p.route = route;
    p.variant = variant;
    p.stages = stages;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(p.name, sizeof p.name, fmt, ap);
    va_end(ap);
    return p;
}

// Device buffers of one tuning run, released on every path out.
struct Scratch {
    std::vector<void*> ptrs;
    cudaStream_t st = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    ~Scratch() {
        if (st) cudaStreamSynchronize(st);
        for (void* p : ptrs) cudaFree(p);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
        if (st) cudaStreamDestroy(st);
    }
    int alloc(void** p, size_t bytes) {
        BYBYCU_CUDA_TRY(cudaMalloc(p, std::max<size_t>(bytes, 16)));
        ptrs.push_back(*p);
        return BYBYCU_OK;
    }
};

int copies_for(size_t weight_bytes) {
    const size_t c = (kColdBytes + weight_bytes - 1) / std::max<size_t>(weight_bytes, 1);
    return static_cast<int>(std::max<size_t>(1, std::min<size_t>(kMaxCopies, c)));
}

// Replicates `n` weight buffers `copies` times: out[c * n + i] is copy c of buffer i
// (copy 0 is the caller's own).
int replicate(Scratch& s, const void* const* bufs, const size_t* bytes, int n, int copies, std::vector<const void*>* out) {
    out->assign(static_cast<size_t>(copies) * n, nullptr);
    for (int i = 0; i < n; ++i) (*out)[i] = bufs[i];
    for (int c = 1; c < copies; ++c)
        for (int i = 0; i < n; ++i) {
            void* p = nullptr;
            if (int rc = s.alloc(&p, bytes[i])) return rc;
            BYBYCU_CUDA_TRY(cudaMemcpyAsync(p, bufs[i], bytes[i], cudaMemcpyDeviceToDevice, s.st));
            (*out)[static_cast<size_t>(c) * n + i] = p;
        }
    return BYBYCU_OK;
}

// Reads and clears the device error word after the stream's work (a candidate whose bounded
// wait ran out is rejected, not fatal).
int take_device_error(uint32_t* code) {
    BYBYCU_CUDA_TRY(cudaMemcpyFromSymbol(code, g_device_error, sizeof *code));
    if (*code) {
        const uint32_t zero = 0;
        BYBYCU_CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof zero));
    }
    return BYBYCU_OK;
}

// The selection loop of vulkanPrepareQ4Tuned (q4_autotune.nim:485-532).  *chosen is set when
// a plan was selected; errors of candidate 0 (the reference) are returned.
int select_plan(const char* what, const Key& key, int M, int N, const std::vector<Cand>& cands, const Runner& run,
                int copies, Scratch& s, float* out, bybycu_plan* chosen, bool* ok) {
    const auto t_start = std::chrono::steady_clock::now();
    *ok = false;
    const size_t n_out = static_cast<size_t>(M) * N;
    std::vector<float> ref(n_out), got(n_out);
    std::vector<int> valid;
    for (size_t i = 0; i < cands.size(); ++i) {
        const bybycu_plan& p = cands[i].plan;
        int rc = run(p, 0, out, s.st);
        if (rc == BYBYCU_OK) {
            const cudaError_t e = cudaStreamSynchronize(s.st);
            rc = e == cudaSuccess ? BYBYCU_OK : cuda_fail(e, "tuning run");
        }
        uint32_t dev_err = 0;
        if (rc == BYBYCU_OK) rc = take_device_error(&dev_err);
        if (rc == BYBYCU_OK && dev_err) rc = set_error(BYBYCU_ERR_DEVICE, "device error %u", dev_err);
        if (rc != BYBYCU_OK) {
            if (i == 0) return rc;
            if (verbose()) {
                char msg[256];
                bybycu_last_error(msg, sizeof msg);
                fprintf(stderr, "[q4-tune:cuda] reject %s: %s\n", p.name, msg);
            }
            cudaGetLastError();
            continue;
        }
        BYBYCU_CUDA_TRY(cudaMemcpy(i == 0 ? ref.data() : got.data(), out, n_out * 4, cudaMemcpyDeviceToHost));
        const std::vector<float>& v = i == 0 ? ref : got;
        bool finite = true;
        for (float f : v) finite = finite && std::isfinite(f);
        if (i == 0) {
            if (!finite) return BYBYCU_OK;   // nothing to compare against
            valid.push_back(0);
            continue;
        }
        float err = 0.0f, mag = 0.0f;
        for (size_t j = 0; j < n_out; ++j) {
            err = std::max(err, std::fabs(v[j] - ref[j]));
            mag = std::max(mag, std::fabs(ref[j]));
        }
        if (finite && err <= std::max(1e-5f, mag * cands[i].tol)) valid.push_back(static_cast<int>(i));
        else if (verbose())
            fprintf(stderr, "[q4-tune:cuda] parity reject %s: err=%g max=%g finite=%d\n", p.name, err, mag, finite);
    }
    if (valid.size() < 2) {   // only the reference ran: keep the built-in choice
        *ok = false;
        return BYBYCU_OK;
    }
    const int reps = M == 1 ? 32 : 8;
    std::vector<std::vector<float>> samples(valid.size());
    for (int round = 0; round < 3; ++round) {
        for (size_t j = 0; j < valid.size(); ++j) {
            const size_t vi = round % 2 == 0 ? j : valid.size() - 1 - j;
            const bybycu_plan& p = cands[valid[vi]].plan;
            tune_hold_kernel<<<1, 32, 0, s.st>>>(1000000ull + 20000ull * reps);
            BYBYCU_LAUNCH_CHECK("tune_hold_kernel");
            BYBYCU_CUDA_TRY(cudaEventRecord(s.e0, s.st));
            for (int r = 0; r < reps; ++r)
                if (int rc = run(p, r % copies, out, s.st)) return rc;
            BYBYCU_CUDA_TRY(cudaEventRecord(s.e1, s.st));
            BYBYCU_CUDA_TRY(cudaEventSynchronize(s.e1));
            float ms = 0.0f;
            BYBYCU_CUDA_TRY(cudaEventElapsedTime(&ms, s.e0, s.e1));
            samples[vi].push_back(ms / reps);
        }
    }
    for (auto& t : samples) std::sort(t.begin(), t.end());
    if (verbose())
        for (size_t j = 0; j < valid.size(); ++j)
            fprintf(stderr, "[q4-tune:cuda]   %-24s %.4f ms (min %.4f, max %.4f)\n", cands[valid[j]].plan.name,
                    static_cast<double>(samples[j][1]), static_cast<double>(samples[j][0]),
                    static_cast<double>(samples[j][2]));
    size_t best = 0;
    for (size_t j = 1; j < valid.size(); ++j)
        if (samples[j][1] < samples[best][1] * 0.97f) best = j;
    *chosen = cands[valid[best]].plan;
    chosen->ms = samples[best][1];
    *ok = true;
    const double wall = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_start).count();
    fprintf(stderr,
            "[q4-tune:cuda] %s %dx%d M=%d: %s %.4fms (reference %.4fms; %zu validated candidates; tuneWall=%.3fs)\n",
            what, key.K, key.N, M, chosen->name, static_cast<double>(chosen->ms), static_cast<double>(samples[0][1]),
            valid.size(), wall);
    return BYBYCU_OK;
}

// Common front: switches, the table, the cache.  Returns true when the caller has nothing
// more to do (*prepared set).
bool lookup_first(const Key& k, const char* what, int M, int* prepared) {
    bybycu_plan p;
    if (find_plan(k, &p)) {
        *prepared = 1;
        return true;
    }
    if (cached_plan(k.device, k, &p)) {
        install(k, p);
        *prepared = 1;
        fprintf(stderr, "[q4-tune:cuda] %s %dx%d M=%d: cache hit %s\n", what, k.K, k.N, M, p.name);
        return true;
    }
    return false;
}

// The table key of a shape as the ABI names it (fields an op does not use are zero).
Key abi_key(int dev, int op, int fmt, int x_dtype, int M, int K, int N, int group_size, int n_groups_per_row) {
    const bool tile = op == BYBYCU_OP_TILE_GEMM;
    return Key{dev, op, tile ? fmt : 0, tile ? x_dtype : BYBYCU_DT_F32, K, N, tile ? 0 : group_size,
               tile ? 0 : n_groups_per_row, mclass_of(M)};
}

}  // namespace tune

void apply_tile_gemm_plan(GemmArgs* a, int* route) {
    using namespace tune;
    if (g_count.load(std::memory_order_acquire) == 0) return;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    bybycu_plan p;
    if (!find_plan(Key{dev, BYBYCU_OP_TILE_GEMM, a->fmt, a->x_dtype, a->K, a->N, 0, 0, mclass_of(a->M)}, &p)) return;
    GemmArgs t = *a;
    t.variant = p.variant;
    t.stages = p.stages;
    const bool runs = p.route == BYBYCU_ROUTE_SIMT || (p.route == BYBYCU_ROUTE_GEMV && gemv_supports(t)) ||
                      (p.route == BYBYCU_ROUTE_TC && tc_supports(t));
    if (!runs) return;
    *a = t;
    *route = p.route;
    g_dispatches.fetch_add(1, std::memory_order_relaxed);
}

void apply_q4_plan(int M, int K, int N, int group, int groups, bool fast, bool tc, int* route, int* stages) {
    using namespace tune;
    if (g_count.load(std::memory_order_acquire) == 0) return;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        cudaGetLastError();
        return;
    }
    bybycu_plan p;
    if (!find_plan(Key{dev, BYBYCU_OP_MATMUL_Q4, 0, BYBYCU_DT_F32, K, N, group, groups, mclass_of(M)}, &p)) return;
    if ((p.route == BYBYCU_ROUTE_GEMV && !fast) || (p.route == BYBYCU_ROUTE_TC && !tc)) return;
    *route = p.route;
    *stages = p.stages;
    g_dispatches.fetch_add(1, std::memory_order_relaxed);
}

}  // namespace bybycu

using namespace bybycu;
using namespace bybycu::tune;

extern "C" {

int bybycu_prepare_tile_gemm_tuned(int fmt, int x_dtype, int M, int K, int N, const void* packed, int64_t packed_len,
                                   int64_t scale_base, int* prepared) {
    if (!prepared) return set_error(BYBYCU_ERR_ARGS, "prepared is NULL");
    *prepared = 0;
    if (!packed) return set_error(BYBYCU_ERR_ARGS, "tile GEMM weights are missing");
    if (fmt != BYBYCU_FMT_FP4KM && fmt != BYBYCU_FMT_F16 && fmt != BYBYCU_FMT_Q4B32)
        return set_error(BYBYCU_ERR_ARGS, "unknown tile format %d", fmt);
    if (x_dtype != BYBYCU_DT_F32 && x_dtype != BYBYCU_DT_BF16)
        return set_error(BYBYCU_ERR_ARGS, "tile GEMM element types must be F32 or BF16");
    const int mc = mclass_of(M);
    if (int rc = check_tile_gemm(fmt, mc, K, N, static_cast<int64_t>(mc) * K, packed_len, scale_base, 272, 0,
                                 static_cast<int64_t>(mc) * N))
        return rc;
    if (env_off("BYBY_Q4_TUNED") || env_off("BYBY_GPU_AUTOTUNE")) return BYBYCU_OK;
    int dev = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    const Key key{dev, BYBYCU_OP_TILE_GEMM, fmt, x_dtype, K, N, 0, 0, mc};
    if (lookup_first(key, "tile_gemm", mc, prepared)) return BYBYCU_OK;
    if (fmt == BYBYCU_FMT_FP4KM) return BYBYCU_OK;   // one route (SIMT): nothing to choose

    // the candidates on probe arguments of the real shape and alignment
    GemmArgs probe;
    probe.fmt = fmt; probe.M = mc; probe.K = K; probe.N = N;
    probe.x_dtype = x_dtype;
    probe.packed = static_cast<const uint8_t*>(packed);
    probe.packed_len = packed_len;
    probe.scale_base = scale_base;
    probe.out_dtype = BYBYCU_DT_F32;
    probe.out_ld = N;
    static const uint8_t* const aligned = reinterpret_cast<const uint8_t*>(uintptr_t(1) << 20);
    probe.x = aligned;
    probe.out = const_cast<uint8_t*>(aligned);
    std::vector<Cand> cands;
    cands.push_back({make_plan(BYBYCU_ROUTE_SIMT, -1, 0, "simt-reference"), 0.0f});
    if (fmt == BYBYCU_FMT_Q4B32 && gemv_supports(probe)) {
        if (mc == 1 && x_dtype == BYBYCU_DT_BF16) {
            static const struct { int mode; const char* tag; } forms[] = {
                {kM1I8, "s8"}, {kM1F16, "f16"}, {kM1Bf16, "bf16"}};
            for (const auto& f : forms) {
                if (f.mode == kM1I8 && K > 32768) continue;   // runs as f16 there
                for (int st : {2, 3})
                    cands.push_back({make_plan(BYBYCU_ROUTE_GEMV, f.mode, st, "gemv-%s-st%d", f.tag, st), kTolNarrow});
            }
        } else if (mc == 1) {   // fp32 rows: the integer mode's two images, or the general kernel's
                                // two bf16 terms (the bf16 operand mode has no fp32 form)
            if (K <= 32768)
                for (int st : {2, 3})
                    cands.push_back({make_plan(BYBYCU_ROUTE_GEMV, kM1I8, st, "gemv-s8x2-st%d", st), kTolNarrow});
            cands.push_back({make_plan(BYBYCU_ROUTE_GEMV, kM1Bf16, 0, "gemv-split"), kTolNarrow});
        } else {
            cands.push_back({make_plan(BYBYCU_ROUTE_GEMV, -1, 0, "gemv-stmax"), kTolNarrow});
            for (int st : {2, 3})
                cands.push_back({make_plan(BYBYCU_ROUTE_GEMV, -1, st, "gemv-st%d", st), kTolNarrow});
        }
    }
    if (fmt == BYBYCU_FMT_F16 && gemv_supports(probe))
        for (int per_sm : {1, 2, 3})
            cands.push_back({make_plan(BYBYCU_ROUTE_GEMV, per_sm, 0, "f16gemv-cta%d", per_sm), kTolNarrow});
    if (tc_supports(probe)) cands.push_back({make_plan(BYBYCU_ROUTE_TC, -1, 0, "tc-pair256x128"), kTolNarrow});
    if (cands.size() == 1) return BYBYCU_OK;

    Scratch s;
    BYBYCU_CUDA_TRY(cudaStreamCreateWithFlags(&s.st, cudaStreamNonBlocking));
    BYBYCU_CUDA_TRY(cudaEventCreate(&s.e0));
    BYBYCU_CUDA_TRY(cudaEventCreate(&s.e1));
    void* x = nullptr;
    float* out = nullptr;
    if (int rc = s.alloc(&x, static_cast<size_t>(mc) * K * 4)) return rc;
    if (int rc = s.alloc(reinterpret_cast<void**>(&out), static_cast<size_t>(mc) * N * 4)) return rc;
    tune_input_kernel<<<256, 256, 0, s.st>>>(x, static_cast<int64_t>(mc) * K, x_dtype == BYBYCU_DT_BF16);
    BYBYCU_LAUNCH_CHECK("tune_input_kernel");
    const size_t wbytes = static_cast<size_t>(packed_len);
    const int copies = copies_for(wbytes);
    std::vector<const void*> wcopy;
    const void* bufs[1] = {packed};
    if (int rc = replicate(s, bufs, &wbytes, 1, copies, &wcopy)) return rc;
    const Runner run = [&](const bybycu_plan& p, int copy, float* o, cudaStream_t st) {
        GemmArgs a = probe;
        a.x = x;
        a.packed = static_cast<const uint8_t*>(wcopy[copy]);
        a.out = o;
        a.stream = st;
        a.variant = p.variant;
        a.stages = p.stages;
        switch (p.route) {
            case BYBYCU_ROUTE_GEMV: return gemv_supports(a) ? launch_gemv(a) : set_error(BYBYCU_ERR_SHAPE, "GEMV");
            case BYBYCU_ROUTE_TC: return tc_supports(a) ? launch_tc(a) : set_error(BYBYCU_ERR_SHAPE, "TC");
            default: return launch_simt(a);
        }
    };
    bybycu_plan best{};
    bool ok = false;
    if (int rc = select_plan("tile_gemm", key, mc, N, cands, run, copies, s, out, &best, &ok)) return rc;
    if (!ok) return BYBYCU_OK;
    install(key, best);
    save_plan(dev, key, best);
    *prepared = 1;
    return BYBYCU_OK;
}

int bybycu_prepare_q4_tuned(const uint8_t* wq, const float* scales, const float* zeros, int M, int K, int N,
                            int group_size, int n_groups_per_row, int* prepared) {
    if (!prepared) return set_error(BYBYCU_ERR_ARGS, "prepared is NULL");
    *prepared = 0;
    if (!wq || !scales || !zeros) return set_error(BYBYCU_ERR_ARGS, "matmul_q4 weights are missing");
    if (M <= 0 || K <= 0 || N <= 0 || group_size < 0)
        return set_error(BYBYCU_ERR_SHAPE, "unsupported matmul_q4 shape M=%d K=%d N=%d", M, K, N);
    const int64_t need = group_size > 0 ? (static_cast<int64_t>(K) + group_size - 1) / group_size : 1;
    if (n_groups_per_row < need)
        return set_error(BYBYCU_ERR_SHAPE, "matmul_q4: %d groups per row, K=%d with group %d needs %lld",
                         n_groups_per_row, K, group_size, static_cast<long long>(need));
    if (env_off("BYBY_Q4_TUNED") || env_off("BYBY_GPU_AUTOTUNE")) return BYBYCU_OK;
    int dev = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    const int mc = mclass_of(M);
    const Key key{dev, BYBYCU_OP_MATMUL_Q4, 0, BYBYCU_DT_F32, K, N, group_size, n_groups_per_row, mc};
    if (lookup_first(key, "matmul_q4", mc, prepared)) return BYBYCU_OK;

    Scratch s;
    BYBYCU_CUDA_TRY(cudaStreamCreateWithFlags(&s.st, cudaStreamNonBlocking));
    BYBYCU_CUDA_TRY(cudaEventCreate(&s.e0));
    BYBYCU_CUDA_TRY(cudaEventCreate(&s.e1));
    float *x = nullptr, *out = nullptr;
    if (int rc = s.alloc(reinterpret_cast<void**>(&x), static_cast<size_t>(mc) * K * 4)) return rc;
    if (int rc = s.alloc(reinterpret_cast<void**>(&out), static_cast<size_t>(mc) * N * 4)) return rc;
    std::vector<Cand> cands;
    cands.push_back({make_plan(BYBYCU_ROUTE_SIMT, -1, 0, "q4-exact-reference"), 0.0f});
    if (q4a_fast_supports(mc, K, N, group_size, n_groups_per_row, x, wq, scales, zeros))
        for (int st : {2, 3})
            cands.push_back({make_plan(BYBYCU_ROUTE_GEMV, -1, st, "q4-s8-decode-st%d", st), kTolNarrow});
    if (mc > 1 && tc_asym_supports(mc, K, N, group_size, n_groups_per_row, x, wq, scales, zeros, out))
        cands.push_back({make_plan(BYBYCU_ROUTE_TC, -1, 0, "q4-tc-pair256x128"), kTolNarrow});
    if (cands.size() == 1) return BYBYCU_OK;
    tune_input_kernel<<<256, 256, 0, s.st>>>(x, static_cast<int64_t>(mc) * K, 0);
    BYBYCU_LAUNCH_CHECK("tune_input_kernel");
    const size_t bytes[3] = {static_cast<size_t>(N) * ((K + 1) / 2), static_cast<size_t>(N) * n_groups_per_row * 4,
                             static_cast<size_t>(N) * n_groups_per_row * 4};
    const int copies = copies_for(bytes[0] + bytes[1] + bytes[2]);
    std::vector<const void*> wcopy;
    const void* bufs[3] = {wq, scales, zeros};
    if (int rc = replicate(s, bufs, bytes, 3, copies, &wcopy)) return rc;
    const Runner run = [&](const bybycu_plan& p, int copy, float* o, cudaStream_t st) -> int {
        const uint8_t* w = static_cast<const uint8_t*>(wcopy[3 * copy]);
        const float* sc = static_cast<const float*>(wcopy[3 * copy + 1]);
        const float* z = static_cast<const float*>(wcopy[3 * copy + 2]);
        if (p.route == BYBYCU_ROUTE_GEMV) return launch_q4a(K, N, x, w, sc, z, o, st, p.stages);
        if (p.route == BYBYCU_ROUTE_TC) return launch_tc_asym(mc, K, N, x, w, sc, z, o, st);
        return bybycu_matmul_q4(x, w, sc, z, o, mc, K, N, group_size, n_groups_per_row, BYBYCU_ROUTE_SIMT, st);
    };
    bybycu_plan best{};
    bool ok = false;
    if (int rc = select_plan("matmul_q4", key, mc, N, cands, run, copies, s, out, &best, &ok)) return rc;
    if (!ok) return BYBYCU_OK;
    install(key, best);
    save_plan(dev, key, best);
    *prepared = 1;
    return BYBYCU_OK;
}

int bybycu_plan_get(int op, int fmt, int x_dtype, int M, int K, int N, int group_size, int n_groups_per_row,
                    bybycu_plan* plan, int* found) {
    if (!plan || !found) return set_error(BYBYCU_ERR_ARGS, "plan_get: NULL output");
    int dev = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    const Key k = abi_key(dev, op, fmt, x_dtype, M, K, N, group_size, n_groups_per_row);
    *found = find_plan(k, plan) ? 1 : 0;
    return BYBYCU_OK;
}

int bybycu_plan_set(int op, int fmt, int x_dtype, int M, int K, int N, int group_size, int n_groups_per_row,
                    const bybycu_plan* plan) {
    if (op != BYBYCU_OP_TILE_GEMM && op != BYBYCU_OP_MATMUL_Q4) return set_error(BYBYCU_ERR_ARGS, "unknown op %d", op);
    if (M <= 0 || K <= 0 || N <= 0) return set_error(BYBYCU_ERR_SHAPE, "plan_set: bad shape M=%d K=%d N=%d", M, K, N);
    if (plan && ((plan->route != BYBYCU_ROUTE_SIMT && plan->route != BYBYCU_ROUTE_GEMV && plan->route != BYBYCU_ROUTE_TC) ||
                 plan->variant < -1 ||
                 plan->stages < 0 || plan->stages > 8))
        return set_error(BYBYCU_ERR_ARGS, "plan_set: route %d variant %d stages %d", plan->route, plan->variant,
                         plan->stages);
    int dev = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    const Key k = abi_key(dev, op, fmt, x_dtype, M, K, N, group_size, n_groups_per_row);
    std::lock_guard<std::mutex> lock(g_mu);
    if (plan) g_plans[k] = *plan;
    else g_plans.erase(k);
    g_count.store(static_cast<int>(g_plans.size()), std::memory_order_release);
    return BYBYCU_OK;
}

int bybycu_plan_clear(void) {
    std::lock_guard<std::mutex> lock(g_mu);
    g_plans.clear();
    g_count.store(0, std::memory_order_release);
    g_dispatches.store(0, std::memory_order_relaxed);
    return BYBYCU_OK;
}

int bybycu_tuning_stats(int* prepared_plans, int64_t* tuned_dispatches) {
    if (prepared_plans) *prepared_plans = g_count.load(std::memory_order_acquire);
    if (tuned_dispatches) *tuned_dispatches = g_dispatches.load(std::memory_order_relaxed);
    return BYBYCU_OK;
}

int bybycu_tune_cache_path(char* buf, int buf_len) {
    if (!buf || buf_len <= 0) return set_error(BYBYCU_ERR_ARGS, "tune_cache_path: no buffer");
    int dev = 0;
    BYBYCU_CUDA_TRY(cudaGetDevice(&dev));
    std::string path;
    if (int rc = cache_path(dev, &path)) return rc;
    snprintf(buf, static_cast<size_t>(buf_len), "%s", path.c_str());
    return BYBYCU_OK;
}

}  // extern "C"
