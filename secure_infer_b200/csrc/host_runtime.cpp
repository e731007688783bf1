// host_runtime.cpp -- host side of the authenticated KV transfer path.
//
// What the reference does per interposed vendor copy (secure_infer.cpp:
// 6290-7116 for H2D, :8076-8562 and :2359-2970 for D2H) is done here per
// layer:
//
//   H2D reload of one layer/kind (n records)
//     host   tickets -> IVs (:274-300) -> AADs (:730-775) -> OpenSSL
//            AES-128-GCM on worker threads into a pinned staging slot laid
//            out as n records C[aligned32] || tag || 0^16 || AAD (:6379-6388)
//     stream one cudaMemcpyAsync of the whole slot
//     producer stream: AES-CTR keystream for all n IVs (depends only on the
//            tickets, so it runs while the ciphertext is still on the link)
//     stream fused kernel: GHASH verify + XOR + (dequant) + scatter into the
//            paged cache, zeroing failed records; status D2H; layer event
//   recovery_wait_layer_authentication(layer): joins the layer's statuses and
//     retries each failed record once from the trusted host copy with a fresh
//     ticket (:7303-7333).
//
//   D2H writeback of one layer/kind (n blocks)
//     stream (quantise) + CTR encrypt + tag on device into a staging slot,
//            one D2H copy of the records
//     host   a completion thread waits for the copy, then worker threads
//            verify + decrypt every record with OpenSSL into the host pool
//            (:2470-2547); a failed record is zeroed and reported.
#include "gcm_kernels.cuh"
#include "kx.cuh"
#include "../../include/secure_infer.h"

#include <openssl/evp.h>
#include <pthread.h>
#include <sched.h>
#include <openssl/rand.h>
#include <openssl/crypto.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <shared_mutex>
#include <thread>
#include <unordered_set>
#include <vector>

namespace sib {
namespace host {
namespace {

constexpr uint64_t kAadBytes = 64;

void store_be32(uint8_t* d, uint32_t v)
{
    d[0] = static_cast<uint8_t>(v >> 24); d[1] = static_cast<uint8_t>(v >> 16);
    d[2] = static_cast<uint8_t>(v >> 8);  d[3] = static_cast<uint8_t>(v);
}

void store_be64(uint8_t* d, uint64_t v)
{
    for (int i = 0; i < 8; ++i) d[i] = static_cast<uint8_t>(v >> (56 - 8 * i));
}

uint32_t load_be32(const uint8_t* s)
{
    return (static_cast<uint32_t>(s[0]) << 24) | (static_cast<uint32_t>(s[1]) << 16) |
           (static_cast<uint32_t>(s[2]) << 8) | s[3];
}

uint64_t aligned32(uint64_t count)
{
    const uint64_t a = (count + 31u) & ~static_cast<uint64_t>(31u);
    return a ? a : 32u;
}

uint64_t record_bytes(uint64_t count) { return aligned32(count) + 32u + kAadBytes; }

uint64_t round16(uint64_t v) { return (v + 15u) & ~static_cast<uint64_t>(15u); }

// ---------------------------------------------------------------- host ranges
struct HostRange {
    uintptr_t begin, end;
    uint32_t layer, kind;
    size_t block_bytes;
};

// Lookups (one per record, from every crypto worker) share the lock;
// registrations take it exclusively.
std::shared_mutex g_ranges_mu;
std::vector<HostRange> g_ranges;

bool lookup_range(const void* p, size_t bytes, HostRange* out, uint64_t* block, uint64_t* offset)
{
    const uintptr_t b = reinterpret_cast<uintptr_t>(p);
    if (bytes > UINTPTR_MAX - b) return false;
    const uintptr_t e = b + bytes;
    std::shared_lock<std::shared_mutex> lock(g_ranges_mu);
    // Newest registration first: a host allocation that reuses the address of
    // a freed, previously registered tensor must get its own metadata.
    for (auto it = g_ranges.rbegin(); it != g_ranges.rend(); ++it) {
        const HostRange& r = *it;
        if (b < r.begin || e > r.end) continue;
        *out = r;
        const uint64_t rel = b - r.begin;
        const uint64_t stride = r.block_bytes ? r.block_bytes : 1u;
        *block = rel / stride;
        *offset = rel % stride;
        return true;
    }
    return false;
}

void build_aad(const void* host_ptr, size_t bytes, uint8_t direction, uint64_t ticket, uint64_t transfer_offset,
               uint64_t epoch, uint8_t out[64])
{
    HostRange r{};
    uint64_t block = 0, offset = 0;
    if (!lookup_range(host_ptr, bytes, &r, &block, &offset)) {
        // Unregistered memory: deterministic descriptor from the address.
        r.layer = UINT32_MAX;
        r.kind = UINT32_MAX;
        block = reinterpret_cast<uintptr_t>(host_ptr);
        offset = 0;
    }
    std::memset(out, 0, 64);
    out[0] = 'S'; out[1] = 'F'; out[2] = 'A'; out[3] = 'D';
    out[4] = 1;
    out[5] = direction;
    out[6] = static_cast<uint8_t>(r.kind & 0xffu);
    store_be32(out + 8, r.layer);
    store_be64(out + 12, block);
    store_be64(out + 20, offset);
    store_be64(out + 28, bytes);
    store_be64(out + 36, ticket);
    store_be64(out + 44, transfer_offset);
    store_be64(out + 52, epoch);
}

// ---------------------------------------------------------------- worker pool
// Restricts the calling thread to `cpus` (best effort: a failure leaves the
// thread where it was).
void pin_self(const std::vector<int>& cpus)
{
    cpu_set_t set;
    CPU_ZERO(&set);
    for (int c : cpus)
        if (c >= 0 && c < CPU_SETSIZE) CPU_SET(c, &set);
    if (CPU_COUNT(&set) > 0) pthread_setaffinity_np(pthread_self(), sizeof(set), &set);
}

class Pool {
public:
    // n workers; with a non-empty `pin`, worker i runs on pin[(i + 1) % size]
    // (pin[0] is left to the calling thread, which works too).
    Pool(unsigned n, const std::vector<int>& pin)
    {
        for (unsigned i = 0; i < n; ++i)
            threads_.emplace_back([this, i, pin] {
                if (!pin.empty()) pin_self({pin[(i + 1) % pin.size()]});
                run();
            });
    }
    ~Pool()
    {
        {
            std::lock_guard<std::mutex> lock(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }
    size_t size() const { return threads_.size(); }

    // Runs fn(0..n-1) on the workers and the calling thread; returns when done.
    void parallel_for(size_t n, const std::function<void(size_t)>& fn)
    {
        if (n == 0) return;
        auto job = std::make_shared<Job>();
        job->n = n;
        job->fn = &fn;
        const size_t helpers = std::min(threads_.size(), n - 1);
        {
            std::lock_guard<std::mutex> lock(mu_);
            for (size_t i = 0; i < helpers; ++i) queue_.push_back(job);
        }
        cv_.notify_all();
        work(*job);
        std::unique_lock<std::mutex> lock(job->mu);
        job->cv.wait(lock, [&] { return job->done == job->n && job->workers == 0; });
    }

private:
    struct Job {
        size_t n = 0;
        const std::function<void(size_t)>* fn = nullptr;
        std::atomic<size_t> next{0};
        size_t done = 0;
        int workers = 0;
        std::mutex mu;
        std::condition_variable cv;
    };

    static void work(Job& job)
    {
        {
            std::lock_guard<std::mutex> lock(job.mu);
            ++job.workers;
        }
        size_t finished = 0;
        for (size_t i = job.next.fetch_add(1); i < job.n; i = job.next.fetch_add(1)) {
            (*job.fn)(i);
            ++finished;
        }
        std::lock_guard<std::mutex> lock(job.mu);
        job.done += finished;
        --job.workers;
        job.cv.notify_all();
    }

    void run()
    {
        for (;;) {
            std::shared_ptr<Job> job;
            {
                std::unique_lock<std::mutex> lock(mu_);
                cv_.wait(lock, [&] { return stop_ || !queue_.empty(); });
                if (stop_ && queue_.empty()) return;
                job = queue_.front();
                queue_.pop_front();
            }
            if (job->next.load() < job->n) work(*job);
        }
    }

    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable cv_;
    std::deque<std::shared_ptr<Job>> queue_;
    bool stop_ = false;
};

// Host cores of this rank.  Ranks that share a host (LOCAL_WORLD_SIZE > 1, as
// torchrun sets it) split the process's CPU affinity set into disjoint equal
// slices, rank LOCAL_RANK taking slice LOCAL_RANK, so that N ranks start N
// small OpenSSL pools instead of N pools as large as the host.  One rank alone
// uses every allowed CPU.  SECURE_INFER_CRYPTO_THREADS overrides the worker
// count, SECURE_INFER_PIN_THREADS=0 turns pinning off (=1 pins a lone rank too).
struct PoolPlan {
    unsigned threads = 0;
    std::vector<int> cpus;   // this rank's slice, in CPU order
    bool pinned = false;
};

unsigned env_unsigned(const char* name, unsigned fallback)
{
    const char* v = std::getenv(name);
    if (v == nullptr || *v == 0) return fallback;
    const int x = std::atoi(v);
    return x < 0 ? fallback : static_cast<unsigned>(x);
}

PoolPlan make_pool_plan()
{
    PoolPlan plan;
    std::vector<int> all;
    cpu_set_t set;
    CPU_ZERO(&set);
    if (sched_getaffinity(0, sizeof(set), &set) == 0) {
        for (int c = 0; c < CPU_SETSIZE; ++c)
            if (CPU_ISSET(c, &set)) all.push_back(c);
    }
    if (all.empty()) {
        const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
        for (unsigned c = 0; c < hw; ++c) all.push_back(static_cast<int>(c));
    }
    const unsigned local_world = std::max(1u, env_unsigned("LOCAL_WORLD_SIZE", 1));
    const unsigned local_rank = std::min(env_unsigned("LOCAL_RANK", 0), local_world - 1);
    const size_t share = std::max<size_t>(1, all.size() / local_world);
    const size_t first = std::min(all.size() - 1, static_cast<size_t>(local_rank) * share);
    plan.cpus.assign(all.begin() + first, all.begin() + std::min(all.size(), first + share));
    // The calling thread encrypts too, so a slice of c cores gets c - 1 workers.
    const unsigned fallback = static_cast<unsigned>(std::min<size_t>(plan.cpus.size() - 1, 31));
    plan.threads = std::getenv("SECURE_INFER_CRYPTO_THREADS") ? env_unsigned("SECURE_INFER_CRYPTO_THREADS", fallback)
                                                              : fallback;
    plan.pinned = env_unsigned("SECURE_INFER_PIN_THREADS", local_world > 1 ? 1u : 0u) != 0;
    return plan;
}

const PoolPlan& pool_plan()
{
    static const PoolPlan plan = make_pool_plan();
    return plan;
}

Pool& pool()
{
    static Pool p(pool_plan().threads, pool_plan().pinned ? pool_plan().cpus : std::vector<int>{});
    return p;
}

// Library threads other than the pool's (D2H verifier, lookahead encryptor)
// stay on the rank's slice when pinning is on.
void pin_library_thread()
{
    if (pool_plan().pinned) pin_self(pool_plan().cpus);
}

// ---------------------------------------------------------------- OpenSSL
// Per-thread AES-128-GCM contexts keyed once per session key: a record then
// only sets its IV (EVP_*Init_ex with key = null keeps the expanded key and
// GHASH table), instead of re-expanding the key for every 10-256 KiB record.
// A session (re)init bumps g_key_generation, which re-keys every context on
// its next use.
std::atomic<uint64_t> g_key_generation{1};

struct KeyedCtx {
    EVP_CIPHER_CTX* ctx = EVP_CIPHER_CTX_new();
    uint64_t generation = 0;
    ~KeyedCtx() { EVP_CIPHER_CTX_free(ctx); }
};

EVP_CIPHER_CTX* keyed_ctx(KeyedCtx& k, const uint8_t key[16], bool encrypt)
{
    const uint64_t gen = g_key_generation.load(std::memory_order_acquire);
    if (k.ctx == nullptr) return nullptr;
    if (k.generation != gen) {
        EVP_CIPHER_CTX_reset(k.ctx);
        const bool ok =
            (encrypt ? EVP_EncryptInit_ex(k.ctx, EVP_aes_128_gcm(), nullptr, nullptr, nullptr)
                     : EVP_DecryptInit_ex(k.ctx, EVP_aes_128_gcm(), nullptr, nullptr, nullptr)) == 1 &&
            EVP_CIPHER_CTX_ctrl(k.ctx, EVP_CTRL_GCM_SET_IVLEN, 12, nullptr) == 1 &&
            (encrypt ? EVP_EncryptInit_ex(k.ctx, nullptr, nullptr, key, nullptr)
                     : EVP_DecryptInit_ex(k.ctx, nullptr, nullptr, key, nullptr)) == 1;
        if (!ok) {
            k.generation = 0;
            return nullptr;
        }
        k.generation = gen;
    }
    return k.ctx;
}

EVP_CIPHER_CTX* thread_enc_ctx(const uint8_t key[16])
{
    thread_local KeyedCtx k;
    return keyed_ctx(k, key, true);
}

EVP_CIPHER_CTX* thread_dec_ctx(const uint8_t key[16])
{
    thread_local KeyedCtx k;
    return keyed_ctx(k, key, false);
}

// Record = C (zero padded to 32) || tag || zero16 || AAD (secure_infer.cpp:6508-6537).
bool encrypt_record(const uint8_t key[16], const uint8_t iv[16], const uint8_t aad[64], const uint8_t* src,
                    uint64_t count, uint8_t* rec)
{
    EVP_CIPHER_CTX* ctx = thread_enc_ctx(key);
    const uint64_t aligned = aligned32(count);
    int n = 0, fin = 0;
    bool ok = ctx != nullptr && EVP_EncryptInit_ex(ctx, nullptr, nullptr, nullptr, iv) == 1 &&
              EVP_EncryptUpdate(ctx, nullptr, &n, aad, static_cast<int>(kAadBytes)) == 1 &&
              EVP_EncryptUpdate(ctx, rec, &n, src, static_cast<int>(count)) == 1 &&
              EVP_EncryptFinal_ex(ctx, rec + n, &fin) == 1 &&
              EVP_CIPHER_CTX_ctrl(ctx, EVP_CTRL_GCM_GET_TAG, 16, rec + aligned) == 1;
    std::memset(rec + count, 0, aligned - count);
    std::memset(rec + aligned + 16, 0, 16);
    std::memcpy(rec + aligned + 32, aad, kAadBytes);
    return ok;
}

// secure_infer.cpp:2479-2501; zeroes `out` on failure.
bool decrypt_record(const uint8_t key[16], const uint8_t iv[16], const uint8_t aad[64], const uint8_t* c,
                    uint64_t count, const uint8_t tag[16], uint8_t* out)
{
    EVP_CIPHER_CTX* ctx = thread_dec_ctx(key);
    int n = 0, fin = 0;
    uint8_t tag_copy[16];
    std::memcpy(tag_copy, tag, 16);
    const bool ok = ctx != nullptr && EVP_DecryptInit_ex(ctx, nullptr, nullptr, nullptr, iv) == 1 &&
                    EVP_DecryptUpdate(ctx, nullptr, &n, aad, static_cast<int>(kAadBytes)) == 1 &&
                    EVP_DecryptUpdate(ctx, out, &n, c, static_cast<int>(count)) == 1 &&
                    EVP_CIPHER_CTX_ctrl(ctx, EVP_CTRL_GCM_SET_TAG, 16, tag_copy) == 1 &&
                    EVP_DecryptFinal_ex(ctx, out + n, &fin) == 1;
    if (!ok) std::memset(out, 0, count);
    return ok;
}

// ---------------------------------------------------------------- session
struct LayerBatch;

// Device launch descriptors for one reload_records call.
struct LaunchSlot {
    uint32_t cap_recs = 0, cap_segs = 0;
    GcmRecord* host_recs = nullptr;
    CtrJob* host_jobs = nullptr;
    GcmRecord* dev_recs = nullptr;
    CtrJob* dev_jobs = nullptr;
    uint4* partials = nullptr;
    uint32_t* counters = nullptr;
    cudaEvent_t free_ev = nullptr;
    bool used = false;
};

// Record staging for one host-side transfer (H2D or D2H).
struct StageSlot {
    uint64_t cap = 0, ks_cap = 0;
    uint32_t cap_recs = 0;
    uint8_t* host = nullptr;       // pinned records
    uint8_t* dev = nullptr;        // device records
    uint8_t* ks = nullptr;         // device keystream
    uint8_t* pkt = nullptr;        // device codec packets (writeback plaintext)
    uint64_t pkt_cap = 0;
    uint8_t* host_aad = nullptr;   // pinned [cap_recs][64] (D2H)
    uint8_t* dev_aad = nullptr;
    const uint8_t** host_ptrs = nullptr;   // pinned [cap_recs] (D2H encode gather)
    const uint8_t** dev_ptrs = nullptr;
    uint32_t* dev_status = nullptr;
    uint32_t* host_status = nullptr;
    cudaEvent_t done = nullptr;
    cudaEvent_t ks_ready = nullptr, copied = nullptr;   // staged reload: keystream / records landed
    std::shared_ptr<LayerBatch> owner;
    std::shared_ptr<struct Prepared> hold;   // pre-encrypted records the slot's copy reads
    bool encrypting = false;       // a submission is encrypting into `host` with the session lock released
};

struct RetryInfo {
    const void* src;
    void* dst;
};

struct LayerBatch {
    uint32_t layer = 0;
    uint64_t job = 0;
    uint32_t n = 0;
    uint64_t count = 0;
    secure_infer_codec codec{};
    bool encrypted = false;
    cudaStream_t stream = nullptr;
    StageSlot* slot = nullptr;
    cudaEvent_t done = nullptr;   // owned
    bool harvested = false;
    std::vector<uint32_t> status;
    std::vector<RetryInfo> items;
    ~LayerBatch()
    {
        if (done) cudaEventDestroy(done);
    }
};

struct D2HGroup {
    uint32_t n = 0;
    uint64_t count = 0;
    StageSlot* slot = nullptr;
    cudaEvent_t copied = nullptr;    // owned
    std::vector<void*> dsts;
    std::vector<uint8_t> ivs;        // [n][16]
    std::vector<uint8_t> aads;       // [n][64]
    bool verified = false;
    bool ok = true;
    uint64_t batch = 0;
};

struct Session {
    bool ready = false;
    int device = 0;
    uint8_t key[16] = {};
    uint8_t salt[4] = {};
    GcmSchedule* sched = nullptr;
    uint32_t rk[44] = {};             // the schedule's round keys, for the layer kernels' parameters
    void* join_tabs = nullptr;        // segment join tables of the layer kernels
    cudaStream_t producer = nullptr;
    cudaStream_t copier = nullptr;    // staged H2D record copies
    // Cross-stream fences of reload_records when the keystream is produced on
    // another stream than the one that consumes it.
    cudaEvent_t consumed_ev = nullptr, produced_ev = nullptr;
    // Tickets handed to callers (secure_infer_new_transfer_ticket, records
    // encrypted by secure_infer_h2d_encrypt_records) and not yet consumed by a
    // pre-encrypted reload.  A given ticket is accepted once: a replay, or a
    // ticket this session never issued, is rejected.  Tickets the library
    // takes for its own staged records are fresh by construction and are not
    // tracked, so the set stays as small as the caller's outstanding records.
    std::mutex replay_mu;
    std::unordered_set<uint64_t> outstanding;

    std::vector<LaunchSlot> launch;   // ring
    size_t launch_next = 0;
    std::vector<StageSlot> h2d;       // ring
    size_t h2d_next = 0;
    // Host side of the staged H2D path: chunks of records are encrypted into
    // a small ring of cached pinned buffers and each chunk is copied as soon
    // as it is complete (see encrypt_ring_locked).
    struct RingChunk {
        uint8_t* host = nullptr;
        uint64_t cap = 0;
        cudaEvent_t ev = nullptr;     // recorded after the chunk's copy
    };
    std::vector<RingChunk> ring;
    uint32_t ring_next = 0;
    std::vector<StageSlot> d2h;       // ring
    size_t d2h_next = 0;
    std::vector<StageSlot> wb;        // ring: scratch of device-resident writebacks
    size_t wb_next = 0;

    std::map<uint32_t, std::vector<std::shared_ptr<LayerBatch>>> pending;
    std::map<uint32_t, cudaEvent_t> last_event;   // not owned: batch->done
    std::map<uint32_t, std::shared_ptr<LayerBatch>> last_batch;
    uint64_t job = 0;

    // D2H completion
    std::deque<std::shared_ptr<D2HGroup>> d2h_queue;
    std::vector<std::shared_ptr<D2HGroup>> d2h_all;
    std::thread d2h_thread;
    std::condition_variable d2h_cv;
    bool d2h_stop = false;

    ~Session()
    {
        // Process exit without secure_infer_session_shutdown(): stop the
        // completion thread without touching CUDA (the runtime may be gone).
        if (d2h_thread.joinable()) {
            d2h_stop = true;
            d2h_cv.notify_all();
            if (d2h_queue.empty()) d2h_thread.join(); else d2h_thread.detach();
        }
    }
};

std::recursive_mutex g_mu;      // H2D path + session state
std::mutex g_events_mu;         // g_s.last_event / last_batch (device-side layer release)
bool host_only_session = false;
std::mutex g_d2h_mu;            // D2H completion state
Session g_s;

std::atomic<uint64_t> g_verified{0}, g_rejected{0}, g_retried{0};
// Transfer tickets come from one counter for the whole process that no session
// (re)init resets, as the reference's process-wide ticket counter
// (secure_infer.cpp:126, :264).  The IV is salt || BE64(ticket) || counter, so
// a counter that restarted at 1 would reuse GCM nonces when a process opens a
// second session with the same key and salt.
std::atomic<uint64_t> g_next_ticket{1};
std::atomic<uint64_t> g_ks_scheduled{0}, g_ks_hit{0}, g_ks_launches{0}, g_generation{0};
// Pre-encryption lookahead (secure_infer_h2d_prepare_layer): records taken
// from a ready entry, reloads that waited for their entry, and reloads that
// found prepared entries outstanding but none of them matching.
std::atomic<uint64_t> g_prep_ready{0}, g_prep_busy{0}, g_prep_missing{0};
std::atomic<uint64_t> g_tamper_h2d_nth{0}, g_tamper_d2h_nth{0};
std::atomic<uint32_t> g_tamper_h2d_target{0};

constexpr size_t kLaunchSlots = 8;

size_t stage_slot_count()
{
    const char* v = std::getenv("SECURE_INFER_STAGE_SLOTS");
    const int n = v ? std::atoi(v) : 3;
    return static_cast<size_t>(std::max(1, std::min(n, 16)));
}

#define CUDA_OK(expr) ((expr) == cudaSuccess)

bool ensure_launch_slot(LaunchSlot& s, uint32_t recs, uint32_t segs)
{
    if (s.used) cudaEventSynchronize(s.free_ev);
    if (s.cap_recs >= recs && s.cap_segs >= segs) return true;
    cudaFreeHost(s.host_recs); cudaFreeHost(s.host_jobs);
    cudaFree(s.dev_recs); cudaFree(s.dev_jobs); cudaFree(s.partials); cudaFree(s.counters);
    s = LaunchSlot{0, 0, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, s.free_ev, false};
    const uint32_t r = std::max<uint32_t>(recs, 256), g = std::max<uint32_t>(segs, 2048);
    if (!CUDA_OK(cudaHostAlloc(&s.host_recs, sizeof(GcmRecord) * r, cudaHostAllocDefault)) ||
        !CUDA_OK(cudaHostAlloc(&s.host_jobs, sizeof(CtrJob) * r, cudaHostAllocDefault)) ||
        !CUDA_OK(cudaMalloc(&s.dev_recs, sizeof(GcmRecord) * r)) ||
        !CUDA_OK(cudaMalloc(&s.dev_jobs, sizeof(CtrJob) * r)) ||
        !CUDA_OK(cudaMalloc(&s.partials, sizeof(uint4) * g)) ||
        !CUDA_OK(cudaMalloc(&s.counters, sizeof(uint32_t) * r)) ||
        !CUDA_OK(cudaMemset(s.counters, 0, sizeof(uint32_t) * r)))
        return false;
    s.cap_recs = r;
    s.cap_segs = g;
    return true;
}

void free_stage(StageSlot& s)
{
    cudaFreeHost(s.host); cudaFreeHost(s.host_aad); cudaFreeHost(s.host_ptrs); cudaFreeHost(s.host_status);
    cudaFree(s.dev); cudaFree(s.ks); cudaFree(s.pkt); cudaFree(s.dev_aad); cudaFree(s.dev_ptrs); cudaFree(s.dev_status);
    s.host = s.dev = s.ks = s.pkt = s.host_aad = s.dev_aad = nullptr;
    s.pkt_cap = 0;
    s.host_ptrs = s.dev_ptrs = nullptr;
    s.host_status = s.dev_status = nullptr;
    s.cap = s.ks_cap = 0;
    s.cap_recs = 0;
}

// H2D staging records are only written by the host and read by the copy
// engine: write-combined pinned memory avoids the read-for-ownership of every
// line the encryption writes (SECURE_INFER_WC_STAGING=0 turns it off).
// H2D record staging: by default a whole layer is encrypted into one staging
// buffer and copied once.  SECURE_INFER_H2D_RING=1 sends records through the
// chunk ring instead: SECURE_INFER_H2D_RING_SLOTS buffers (default 8) of about
// SECURE_INFER_H2D_RING_CHUNK bytes (default 8 MiB), which bounds pinned
// staging memory independently of the layer size.  On a 16-core host the two
// reach the same end-to-end rate with 8 MiB chunks; smaller chunks are slower.
bool h2d_ring()
{
    static const bool on = [] {
        const char* v = std::getenv("SECURE_INFER_H2D_RING");
        return v != nullptr && std::atoi(v) != 0;
    }();
    return on;
}

uint32_t ring_slots()
{
    static const uint32_t n = [] {
        const char* v = std::getenv("SECURE_INFER_H2D_RING_SLOTS");
        const long x = v ? std::atol(v) : 8;
        return static_cast<uint32_t>(std::min<long>(std::max<long>(x, 2), 64));
    }();
    return n;
}

uint64_t ring_chunk_bytes()
{
    static const uint64_t n = [] {
        const char* v = std::getenv("SECURE_INFER_H2D_RING_CHUNK");
        const long long x = v ? std::atoll(v) : (8ll << 20);
        return static_cast<uint64_t>(std::min<long long>(std::max<long long>(x, 64ll << 10), 256ll << 20));
    }();
    return n;
}

bool wc_staging()
{
    static const bool on = [] {
        const char* v = std::getenv("SECURE_INFER_WC_STAGING");
        return v == nullptr || std::atoi(v) != 0;
    }();
    return on;
}

bool ensure_stage(StageSlot& s, uint64_t bytes, uint64_t ks_bytes, uint32_t recs, uint64_t pkt_bytes = 0,
                  bool host_write_only = false)
{
    if (s.cap >= bytes && s.ks_cap >= ks_bytes && s.cap_recs >= recs && s.pkt_cap >= pkt_bytes) return true;
    if (s.done) cudaEventSynchronize(s.done);
    free_stage(s);
    const uint32_t r = std::max<uint32_t>(recs, 256);
    const unsigned host_flags = host_write_only && wc_staging() ? cudaHostAllocWriteCombined : cudaHostAllocDefault;
    if (!CUDA_OK(cudaHostAlloc(&s.host, bytes, host_flags)) || !CUDA_OK(cudaMalloc(&s.dev, bytes)) ||
        (ks_bytes && !CUDA_OK(cudaMalloc(&s.ks, ks_bytes))) ||
        (pkt_bytes && !CUDA_OK(cudaMalloc(&s.pkt, pkt_bytes))) ||
        !CUDA_OK(cudaHostAlloc(&s.host_aad, 64ull * r, cudaHostAllocDefault)) ||
        !CUDA_OK(cudaMalloc(&s.dev_aad, 64ull * r)) ||
        !CUDA_OK(cudaHostAlloc(reinterpret_cast<void**>(&s.host_ptrs), sizeof(void*) * r, cudaHostAllocDefault)) ||
        !CUDA_OK(cudaMalloc(reinterpret_cast<void**>(&s.dev_ptrs), sizeof(void*) * r)) ||
        !CUDA_OK(cudaHostAlloc(reinterpret_cast<void**>(&s.host_status), sizeof(uint32_t) * r, cudaHostAllocDefault)) ||
        !CUDA_OK(cudaMalloc(reinterpret_cast<void**>(&s.dev_status), sizeof(uint32_t) * r))) {
        free_stage(s);
        return false;
    }
    s.cap = bytes;
    s.ks_cap = ks_bytes;
    s.pkt_cap = pkt_bytes;
    s.cap_recs = r;
    return true;
}

void harvest(LayerBatch& b)
{
    if (b.harvested) return;
    cudaEventSynchronize(b.done);
    b.status.assign(b.slot->host_status, b.slot->host_status + b.n);
    b.harvested = true;
}

// n consecutive fresh tickets for the library's own records.
void reserve_tickets(uint32_t n, uint64_t* out)
{
    const uint64_t first = g_next_ticket.fetch_add(n, std::memory_order_relaxed);
    for (uint32_t i = 0; i < n; ++i) out[i] = first + i;
}

// n fresh tickets handed to a caller, redeemable once by reserve_given_ticket.
void issue_tickets(uint32_t n, uint64_t* out)
{
    const uint64_t first = g_next_ticket.fetch_add(n, std::memory_order_relaxed);
    std::lock_guard<std::mutex> lock(g_s.replay_mu);
    for (uint32_t i = 0; i < n; ++i) {
        out[i] = first + i;
        g_s.outstanding.insert(first + i);
    }
}

// A caller-supplied ticket: accepted once (secure_infer.cpp:777-789 rejects
// replays the same way).
bool reserve_given_ticket(uint64_t t)
{
    if (t == 0) return false;
    std::lock_guard<std::mutex> lock(g_s.replay_mu);
    return g_s.outstanding.erase(t) == 1;
}

void iv_for_salt(const uint8_t salt[4], uint64_t ticket, uint8_t iv[16])
{
    std::memcpy(iv, salt, 4);
    store_be64(iv + 4, ticket);   // session nonce 0 in GCM mode (secure_infer.cpp:242-245)
    store_be32(iv + 12, 2u);
}

void iv_for(uint64_t ticket, uint8_t iv[16]) { iv_for_salt(g_s.salt, ticket, iv); }

void iv_words_for(uint64_t ticket, uint32_t w[4])
{
    w[0] = load_be32(g_s.salt);
    w[1] = static_cast<uint32_t>(ticket >> 32);
    w[2] = static_cast<uint32_t>(ticket);
    w[3] = 2u;
}

bool codec_geometry(const secure_infer_codec* codec, CodecParams* cp, uint64_t* packet, bool kv_pair = false)
{
    *cp = CodecParams{};
    *packet = 0;
    if (codec == nullptr || codec->bits == 0) return true;
    const uint32_t max_kind = kv_pair ? SECURE_INFER_KIND_KV : 1u;
    if ((codec->bits != 8 && codec->bits != 4) || codec->kind > max_kind || codec->heads == 0 || codec->heads > 16)
        return false;
    const uint64_t elements = 128ull * codec->heads * 128ull;
    cp->bits = codec->bits;
    cp->kind = codec->kind;
    cp->heads = codec->heads;
    cp->qb = static_cast<uint32_t>(elements * codec->bits / 8);
    cp->sb = static_cast<uint32_t>(elements / 64 * 4);
    *packet = (cp->qb + 2ull * cp->sb + 16 + 15) / 16 * 16;
    return true;
}

bool misaligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

// Keystream for n records (stride layer_ks_stride(count), E_K(J0) in each
// record's last 16 bytes) on `stream`.  Caller holds g_mu.
int keystream_records_locked(const uint64_t* tickets, uint32_t n, uint64_t count, uint8_t* keystream,
                             cudaStream_t stream)
{
    if (!g_s.ready || tickets == nullptr || n == 0 || count == 0 || keystream == nullptr) return -1;
    const uint64_t ks_stride = layer_ks_stride(count);
    std::vector<LayerRec> recs(std::min<uint32_t>(n, kLayerCapLarge));
    for (uint32_t first = 0; first < n; first += kLayerCapLarge) {
        const uint32_t m = std::min<uint32_t>(n - first, kLayerCapLarge);
        LayerHeader h{};
        std::memcpy(h.rk, g_s.rk, sizeof(h.rk));
        h.sched = g_s.sched;
        h.count = count;
        h.ks = keystream + first * ks_stride;
        h.ks_stride = ks_stride;
        h.iv0 = load_be32(g_s.salt);
        h.n = m;
        h.unaligned = misaligned(keystream) ? 1u : 0u;
        for (uint32_t i = 0; i < m; ++i) recs[i] = LayerRec{nullptr, tickets[first + i]};
        if (launch_layer_keystream(h, recs.data(), stream) != cudaSuccess) return -1;
    }
    g_ks_scheduled += n;
    ++g_ks_launches;
    return 0;
}

// Fused verify / XOR / (dequant) / scatter over n device-resident records.
// Raw records with a keystream run on the layer kernel (descriptors in kernel
// parameters); codec records and keystream-less requests use the CTA-segment
// kernel.  Caller holds g_mu.
int verify_records_locked(const uint8_t* records, uint64_t stride, uint64_t count, uint32_t n,
                          const uint64_t* tickets, void* const* dsts, const uint8_t* keystream, uint32_t* status,
                          const secure_infer_codec* codec, cudaStream_t stream)
{
    if (!g_s.ready || records == nullptr || n == 0 || count == 0 || tickets == nullptr || dsts == nullptr ||
        status == nullptr || stride < record_bytes(count) || (stride & 15u))
        return -1;
    CodecParams cp;
    uint64_t packet = 0;
    if (!codec_geometry(codec, &cp, &packet, true)) return -1;
    if (cp.bits && (count != packet || keystream == nullptr)) return -1;
    if (cp.bits && cp.kind == SECURE_INFER_KIND_KV && (n & 1u)) return -1;
    const uint64_t aligned = aligned32(count);
    const uint64_t ks_stride = layer_ks_stride(count);
    const bool rec_misaligned = misaligned(records);

    if (keystream) {
        std::vector<LayerRec> recs(std::min<uint32_t>(n, kLayerCapLarge));
        for (uint32_t first = 0; first < n; first += kLayerCapLarge) {
            const uint32_t m = std::min<uint32_t>(n - first, kLayerCapLarge);
            uint32_t seg_steps = 0, nseg = 0;
            layer_segments_for(count, m, cp.bits, &seg_steps, &nseg);
            LaunchSlot& slot = g_s.launch[g_s.launch_next];
            g_s.launch_next = (g_s.launch_next + 1) % g_s.launch.size();
            if (!ensure_launch_slot(slot, m, nseg * m)) return -1;
            LayerHeader h{};
            std::memcpy(h.rk, g_s.rk, sizeof(h.rk));
        std::memcpy(h.rk, g_s.rk, sizeof(h.rk));
            h.sched = g_s.sched;
            h.records = records + first * stride;
            h.stride = stride;
            h.count = count;
            h.ks = const_cast<uint8_t*>(keystream) + first * ks_stride;
            h.ks_stride = ks_stride;
            h.status = status + first;
            h.partials = slot.partials;
            h.counters = slot.counters;
            h.iv0 = load_be32(g_s.salt);
            h.n = m;
            h.nseg = nseg;
            h.seg_steps = seg_steps;
            h.join_pow = sib::join_tables_for(g_s.join_tabs, seg_steps);
            h.codec = cp;
            // Records of this chunk from index v_first on are V packets.
            const uint32_t v_global = cp.kind == SECURE_INFER_KIND_KV ? n / 2 : (cp.kind == 1 ? 0u : n);
            h.v_first = v_global > first ? std::min<uint32_t>(v_global - first, m) : 0u;
            bool unaligned = rec_misaligned || misaligned(keystream);
            for (uint32_t i = 0; i < m; ++i) {
                recs[i] = LayerRec{static_cast<uint8_t*>(dsts[first + i]), tickets[first + i]};
                unaligned = unaligned || misaligned(dsts[first + i]);
            }
            // Codec packets are read with 16-byte loads and decoded with
            // 16-byte stores: they need aligned records, keystream and blocks.
            if (cp.bits && unaligned) return -1;
            h.unaligned = unaligned ? 1u : 0u;
            if (launch_layer_verify(h, recs.data(), stream) != cudaSuccess) return -1;
            cudaEventRecord(slot.free_ev, stream);
            slot.used = true;
        }
        g_ks_hit += n;
        return 0;
    }

    // No keystream buffer, raw and 16-byte aligned records and destinations:
    // one fused layer kernel computes the keystream itself.
    bool dsts_aligned = !rec_misaligned;
    for (uint32_t i = 0; dsts_aligned && i < n; ++i) dsts_aligned = !misaligned(dsts[i]);
    if (!cp.bits && dsts_aligned) {
        std::vector<LayerRec> recs(std::min<uint32_t>(n, kLayerCapLarge));
        for (uint32_t first = 0; first < n; first += kLayerCapLarge) {
            const uint32_t m = std::min<uint32_t>(n - first, kLayerCapLarge);
            uint32_t seg_steps = 0, nseg = 0;
            layer_segments_for(count, m, 0, &seg_steps, &nseg);
            LaunchSlot& slot = g_s.launch[g_s.launch_next];
            g_s.launch_next = (g_s.launch_next + 1) % g_s.launch.size();
            if (!ensure_launch_slot(slot, m, nseg * m)) return -1;
            LayerHeader h{};
            std::memcpy(h.rk, g_s.rk, sizeof(h.rk));
        std::memcpy(h.rk, g_s.rk, sizeof(h.rk));
            h.sched = g_s.sched;
            h.records = records + first * stride;
            h.stride = stride;
            h.count = count;
            h.status = status + first;
            h.partials = slot.partials;
            h.counters = slot.counters;
            h.iv0 = load_be32(g_s.salt);
            h.n = m;
            h.nseg = nseg;
            h.seg_steps = seg_steps;
            h.join_pow = sib::join_tables_for(g_s.join_tabs, seg_steps);
            for (uint32_t i = 0; i < m; ++i) recs[i] = LayerRec{static_cast<uint8_t*>(dsts[first + i]), tickets[first + i]};
            if (launch_layer_verify_inline(h, recs.data(), stream) != cudaSuccess) return -1;
            cudaEventRecord(slot.free_ev, stream);
            slot.used = true;
        }
        return 0;
    }

    const uint32_t seg_blocks = segment_blocks_for(
        static_cast<uint64_t>(n) * ((kAadBytes + 15u) / 16u + (count + 15u) / 16u + 1u));
    const uint32_t nseg = segments_for(count, kAadBytes, seg_blocks);
    LaunchSlot& slot = g_s.launch[g_s.launch_next];
    g_s.launch_next = (g_s.launch_next + 1) % g_s.launch.size();
    if (!ensure_launch_slot(slot, n, nseg * n)) return -1;
    for (uint32_t i = 0; i < n; ++i) {
        const uint8_t* base = records + i * stride;
        GcmRecord& r = slot.host_recs[i];
        r = GcmRecord{};
        r.op = kOpDecrypt;
        r.in = base;
        r.ks = keystream ? keystream + i * ks_stride : nullptr;
        r.aad = base + aligned + 32;
        r.aad_bytes = static_cast<uint32_t>(kAadBytes);
        r.tag_in = base + aligned;
        r.out = static_cast<uint8_t*>(dsts[i]);
        r.status = status + i;
        r.count = count;
        iv_words_for(tickets[i], r.iv);
        r.seg_first = i * nseg;
        r.nseg = nseg;
        if (rec_misaligned || misaligned(dsts[i]) || misaligned(r.ks)) r.flags |= kRecUnaligned;
    }
    if (!CUDA_OK(cudaMemcpyAsync(slot.dev_recs, slot.host_recs, sizeof(GcmRecord) * n, cudaMemcpyHostToDevice, stream)))
        return -1;
    SegmentLaunch L{};
    L.sched = g_s.sched;
    L.recs = slot.dev_recs;
    L.nrec = n;
    L.total_segs = nseg * n;
    L.partials = slot.partials;
    L.counters = slot.counters;
    L.seg_blocks = seg_blocks;
    if (launch_segments(L, keystream == nullptr, stream) != cudaSuccess) return -1;
    cudaEventRecord(slot.free_ev, stream);
    slot.used = true;
    if (keystream) g_ks_hit += n;
    return 0;
}

// Keystream on `producer`, joined into `stream`, then the fused kernel.
int reload_records_locked(uint32_t layer, const uint8_t* records, uint64_t stride, uint64_t count, uint32_t n,
                          const uint64_t* tickets, void* const* dsts, uint8_t* keystream, uint32_t* status,
                          const secure_infer_codec* codec, cudaStream_t stream, cudaStream_t producer)
{
    (void)layer;
    if (keystream) {
        // The caller may reuse one keystream buffer for every call: on a
        // separate producer stream the keystream launch first waits for the
        // consumer stream's earlier work (the previous verify reading it).
        const bool cross = producer != stream;
        if (cross && (!CUDA_OK(cudaEventRecord(g_s.consumed_ev, stream)) ||
                      !CUDA_OK(cudaStreamWaitEvent(producer, g_s.consumed_ev, 0))))
            return -1;
        if (keystream_records_locked(tickets, n, count, keystream, producer) != 0) return -1;
        if (cross && (!CUDA_OK(cudaEventRecord(g_s.produced_ev, producer)) ||
                      !CUDA_OK(cudaStreamWaitEvent(stream, g_s.produced_ev, 0))))
            return -1;
    }
    return verify_records_locked(records, stride, count, n, tickets, dsts, keystream, status, codec, stream);
}

void maybe_tamper_h2d(uint8_t* rec, uint64_t count)
{
    uint64_t nth = g_tamper_h2d_nth.load();
    while (nth != 0) {
        if (g_tamper_h2d_nth.compare_exchange_weak(nth, nth - 1)) {
            if (nth == 1) {
                // Flip one byte after host encryption, before the DMA (secure_infer.cpp:6560-6602).
                uint8_t* target = g_tamper_h2d_target.load() == 1 ? rec + aligned32(count) : rec + count / 2;
                target[0] ^= 0x01;
            }
            return;
        }
    }
}

// Encrypts n records (tickets given) into the chunk ring and copies every
// chunk to dev (record i at dev + i * stride) on the copy stream as soon as
// its last record is encrypted, so the copy engine reads freshly written
// lines and the ring's few megabytes are reused instead of a whole layer of
// staging.  Records are taken in increasing order by the pool; a worker that
// needs a ring buffer first waits until the chunk that used it R chunks
// earlier has been copied.  Every record of that chunk was taken before, so
// the wait always ends.  Caller holds g_mu.
bool encrypt_ring_locked(const uint64_t* tickets, const void* const* srcs, uint32_t n, uint64_t count, uint64_t stride,
                         uint8_t* dev)
{
    const uint32_t R = ring_slots();
    const uint64_t per = std::max<uint64_t>(1, ring_chunk_bytes() / stride);
    const uint32_t C = static_cast<uint32_t>(std::min<uint64_t>(per, n));
    const uint32_t chunks = (n + C - 1) / C;
    if (g_s.ring.size() != R) g_s.ring.resize(R);
    for (auto& rc : g_s.ring) {
        if (!rc.ev && !CUDA_OK(cudaEventCreateWithFlags(&rc.ev, cudaEventDisableTiming))) return false;
        if (rc.cap < C * stride) {
            cudaEventSynchronize(rc.ev);
            if (rc.host) cudaFreeHost(rc.host);
            rc.host = nullptr;
            rc.cap = 0;
            if (!CUDA_OK(cudaHostAlloc(&rc.host, C * stride,
                                       wc_staging() ? cudaHostAllocWriteCombined : cudaHostAllocDefault)))
                return false;
            rc.cap = C * stride;
        }
    }
    const uint32_t base = g_s.ring_next;
    std::unique_ptr<std::atomic<uint32_t>[]> left(new std::atomic<uint32_t>[chunks]);
    std::unique_ptr<std::atomic<bool>[]> issued(new std::atomic<bool>[chunks]);
    // Per chunk: 0 = buffer not yet claimed, 1 = one worker is waiting for
    // the buffer's previous copy, 2 = buffer free.  One driver wait per
    // chunk: concurrent event waits from every worker serialise in the driver.
    std::unique_ptr<std::atomic<int>[]> state(new std::atomic<int>[chunks]);
    for (uint32_t k = 0; k < chunks; ++k) {
        left[k] = std::min<uint32_t>(C, n - k * C);
        issued[k] = false;
        state[k] = 0;
    }
    std::mutex mu;
    std::condition_variable cv;
    std::atomic<bool> ok{true};
    const uint8_t* key = g_s.key;
    pool().parallel_for(n, [&](size_t i) {
        const uint32_t k = static_cast<uint32_t>(i / C);
        Session::RingChunk& rc = g_s.ring[(base + k) % R];
        int expect = 0;
        if (state[k].compare_exchange_strong(expect, 1)) {
            if (k >= R) {
                std::unique_lock<std::mutex> lock(mu);
                cv.wait(lock, [&] { return issued[k - R].load(); });
            }
            cudaEventSynchronize(rc.ev);
            {
                std::lock_guard<std::mutex> lock(mu);
                state[k] = 2;
            }
            cv.notify_all();
        } else if (state[k].load() != 2) {
            std::unique_lock<std::mutex> lock(mu);
            cv.wait(lock, [&] { return state[k].load() == 2; });
        }
        uint8_t* rec = rc.host + (i - static_cast<size_t>(k) * C) * stride;
        uint8_t iv[16], aad[64];
        iv_for(tickets[i], iv);
        build_aad(srcs[i], count, SECURE_INFER_DIRECTION_H2D, tickets[i], 0, 0, aad);
        if (!encrypt_record(key, iv, aad, static_cast<const uint8_t*>(srcs[i]), count, rec)) ok = false;
        maybe_tamper_h2d(rec, count);
        if (left[k].fetch_sub(1) == 1) {
            const uint32_t first = k * C, cnt = std::min<uint32_t>(C, n - first);
            if (!CUDA_OK(cudaMemcpyAsync(dev + first * stride, rc.host, cnt * stride, cudaMemcpyHostToDevice,
                                         g_s.copier)) ||
                !CUDA_OK(cudaEventRecord(rc.ev, g_s.copier)))
                ok = false;
            {
                std::lock_guard<std::mutex> lock(mu);
                issued[k] = true;
            }
            cv.notify_all();
        }
    });
    g_s.ring_next = (base + chunks) % R;
    return ok;
}

// ------------------------------------------------------------ lookahead
// Host pre-encryption of a reload the caller announces ahead of time (the
// reference's CPU ciphertext pool, secure_infer.cpp:3264-3710, fed by its
// history predictor; here the caller names the transfer).  Tickets, IVs and
// AADs are fixed when the reload is announced; a background thread encrypts
// the records on the worker pool into a pinned buffer of the prepared pool;
// the matching reload copies that buffer instead of encrypting.
struct Prepared {
    uint32_t layer = 0;
    std::vector<const void*> srcs;
    uint64_t count = 0, stride = 0, generation = 0;
    bool has_codec = false;
    secure_infer_codec codec{};
    std::vector<uint64_t> tickets;
    std::vector<uint8_t> ivs, aads;   // [n][16], [n][64]
    uint8_t key[16] = {};
    uint8_t* host = nullptr;          // pinned [n][stride], from the prepared pool
    uint64_t bytes = 0;
    int state = 0;                    // 0 queued, 1 encrypting, 2 ready, 3 failed (guarded by g_prep.mu)
};

struct PrepPool {
    std::mutex mu;
    std::condition_variable cv;
    std::deque<std::shared_ptr<Prepared>> queue;     // waiting for the encrypt thread
    std::vector<std::shared_ptr<Prepared>> entries;  // announced, not yet taken by a reload
    std::multimap<uint64_t, uint8_t*> free_bufs;      // pinned buffers by size
    uint64_t held = 0;                                // bytes of all pinned buffers
    std::thread worker;
    bool stop = false;

    ~PrepPool()
    {
        // Process exit without secure_infer_session_shutdown(): stop the
        // encryption thread and let it go (it may be inside OpenSSL).
        if (worker.joinable()) {
            {
                std::lock_guard<std::mutex> lock(mu);
                stop = true;
            }
            cv.notify_all();
            worker.detach();
        }
    }
} g_prep;

uint64_t prep_pool_cap()
{
    static const uint64_t cap = [] {
        const char* v = std::getenv("SECURE_INFER_PREPARE_POOL_BYTES");
        const long long x = v ? std::atoll(v) : (256ll << 20);
        return static_cast<uint64_t>(std::max<long long>(x, 0));
    }();
    return cap;
}

// Caller holds g_prep.mu.
void prep_release_locked(Prepared& e)
{
    if (e.host) g_prep.free_bufs.emplace(e.bytes, e.host);
    e.host = nullptr;
}

// A pinned buffer of at least `bytes` from the pool, evicting ready entries
// (oldest first) when the cap would be exceeded.  Caller holds g_prep.mu.
uint8_t* prep_buffer_locked(uint64_t bytes, uint64_t* got)
{
    for (;;) {
        auto it = g_prep.free_bufs.lower_bound(bytes);
        if (it != g_prep.free_bufs.end()) {
            uint8_t* p = it->second;
            *got = it->first;
            g_prep.free_bufs.erase(it);
            return p;
        }
        if (g_prep.held + bytes <= prep_pool_cap()) {
            uint8_t* p = nullptr;
            if (!CUDA_OK(cudaHostAlloc(&p, bytes, wc_staging() ? cudaHostAllocWriteCombined : cudaHostAllocDefault)))
                return nullptr;
            g_prep.held += bytes;
            *got = bytes;
            return p;
        }
        if (!g_prep.free_bufs.empty()) {          // too small: give one back and retry
            auto f = g_prep.free_bufs.begin();
            cudaFreeHost(f->second);
            g_prep.held -= f->first;
            g_prep.free_bufs.erase(f);
            continue;
        }
        auto victim = std::find_if(g_prep.entries.begin(), g_prep.entries.end(),
                                   [](const std::shared_ptr<Prepared>& e) { return e->state >= 2; });
        if (victim == g_prep.entries.end()) return nullptr;
        prep_release_locked(**victim);
        g_prep.entries.erase(victim);
    }
}

void prep_worker()
{
    pin_library_thread();
    for (;;) {
        std::shared_ptr<Prepared> e;
        {
            std::unique_lock<std::mutex> lock(g_prep.mu);
            g_prep.cv.wait(lock, [] { return g_prep.stop || !g_prep.queue.empty(); });
            if (g_prep.stop) return;
            e = g_prep.queue.front();
            g_prep.queue.pop_front();
            if (e->generation != g_generation.load() || e->host == nullptr) {
                e->state = 3;
                g_prep.cv.notify_all();
                continue;
            }
            e->state = 1;
        }
        std::atomic<bool> ok{true};
        const uint32_t n = static_cast<uint32_t>(e->srcs.size());
        pool().parallel_for(n, [&](size_t i) {
            if (!encrypt_record(e->key, &e->ivs[16 * i], &e->aads[64 * i], static_cast<const uint8_t*>(e->srcs[i]),
                                e->count, e->host + i * e->stride))
                ok = false;
        });
        {
            std::lock_guard<std::mutex> lock(g_prep.mu);
            e->state = ok ? 2 : 3;
        }
        g_prep.cv.notify_all();
    }
}

bool same_codec(const Prepared& e, const secure_infer_codec* codec)
{
    if (!codec) return !e.has_codec;
    return e.has_codec && std::memcmp(&e.codec, codec, sizeof(secure_infer_codec)) == 0;
}

// The announced entry for this reload, removed from the pool and complete
// (ready or failed), or null.  Caller holds g_mu.
std::shared_ptr<Prepared> take_prepared(uint32_t layer, const void* const* srcs, uint32_t n, uint64_t count,
                                        const secure_infer_codec* codec)
{
    std::unique_lock<std::mutex> lock(g_prep.mu);
    if (g_prep.entries.empty()) return nullptr;
    const uint64_t gen = g_generation.load();
    auto it = std::find_if(g_prep.entries.begin(), g_prep.entries.end(), [&](const std::shared_ptr<Prepared>& e) {
        return e->layer == layer && e->count == count && e->srcs.size() == n && e->generation == gen &&
               same_codec(*e, codec) && std::equal(e->srcs.begin(), e->srcs.end(), srcs);
    });
    if (it == g_prep.entries.end()) {
        ++g_prep_missing;
        return nullptr;
    }
    std::shared_ptr<Prepared> e = *it;
    g_prep.entries.erase(it);
    if (e->state < 2) {
        ++g_prep_busy;
        g_prep.cv.wait(lock, [&] { return e->state >= 2; });
    }
    if (e->state != 2) {
        prep_release_locked(*e);
        return nullptr;
    }
    return e;
}

// Drops every entry that is not being encrypted right now (those are dropped
// when taken or when the thread finds them stale).
void prep_drop_stale()
{
    std::lock_guard<std::mutex> lock(g_prep.mu);
    const uint64_t gen = g_generation.load();
    for (auto it = g_prep.entries.begin(); it != g_prep.entries.end();) {
        if ((*it)->generation != gen && (*it)->state != 1) {
            if ((*it)->state == 0) (*it)->state = 3;
            prep_release_locked(**it);
            it = g_prep.entries.erase(it);
        } else {
            ++it;
        }
    }
    g_prep.cv.notify_all();
}

// Stops the encrypt thread (after its current entry) and frees the pool,
// including the buffers staging slots still hold.  Call after the device is
// idle: a held buffer may be the source of a copy until then.
void prep_shutdown()
{
    {
        std::lock_guard<std::mutex> lock(g_prep.mu);
        g_prep.stop = true;
    }
    g_prep.cv.notify_all();
    if (g_prep.worker.joinable()) g_prep.worker.join();
    std::lock_guard<std::mutex> lock(g_prep.mu);
    for (auto& slot : g_s.h2d) {
        if (slot.hold) prep_release_locked(*slot.hold);
        slot.hold.reset();
    }
    for (auto& e : g_prep.entries) prep_release_locked(*e);
    for (auto& e : g_prep.queue) prep_release_locked(*e);
    g_prep.entries.clear();
    g_prep.queue.clear();
    for (auto& f : g_prep.free_bufs) cudaFreeHost(f.second);
    g_prep.free_bufs.clear();
    g_prep.held = 0;
    g_prep.stop = false;
}

// Encrypt + stage + device reload.  Returns the batch (not yet registered).
// Notified when a submission stops encrypting into its staging slot.
std::condition_variable_any g_slot_cv;

// Caller holds g_mu.  With `held` (the caller's own, non-recursive hold of
// g_mu) the host encryption runs with the session lock released: the slot is
// marked `encrypting` so no other submission takes it, and authentication
// waits, device-side releases and other submissions proceed meanwhile.
std::shared_ptr<LayerBatch> submit_layer_locked(uint32_t layer, const void* const* srcs, void* const* dsts, uint32_t n,
                                                uint64_t count, const secure_infer_codec* codec, bool encrypted,
                                                const uint64_t* given_tickets, cudaStream_t stream,
                                                std::unique_lock<std::recursive_mutex>* held = nullptr)
{
    if (!g_s.ready || srcs == nullptr || dsts == nullptr || n == 0 || count == 0) return nullptr;
    CodecParams cp;
    uint64_t packet = 0;
    if (!codec_geometry(codec, &cp, &packet, true)) return nullptr;
    if (cp.bits && cp.kind == SECURE_INFER_KIND_KV && (n & 1u)) return nullptr;
    const uint64_t stride = record_bytes(count);
    // The next staging slot that no submission is encrypting into.
    StageSlot* pick = nullptr;
    for (;;) {
        for (size_t t = 0; t < g_s.h2d.size() && pick == nullptr; ++t) {
            const size_t i = (g_s.h2d_next + t) % g_s.h2d.size();
            if (!g_s.h2d[i].encrypting) {
                pick = &g_s.h2d[i];
                g_s.h2d_next = (i + 1) % g_s.h2d.size();
            }
        }
        if (pick != nullptr) break;
        if (held == nullptr) return nullptr;    // every slot is being filled by a submission that released the lock
        g_slot_cv.wait(*held);
        if (!g_s.ready) return nullptr;
    }
    StageSlot& slot = *pick;
    // The slot's previous batch must finish before its buffers are reused;
    // with the lock released, reserved against other submissions, while the
    // GPU gets there.  The batch (slot.owner) keeps its event alive.
    if (held != nullptr && slot.done != nullptr && cudaEventQuery(slot.done) == cudaErrorNotReady) {
        const cudaEvent_t prev = slot.done;
        slot.encrypting = true;
        held->unlock();
        cudaEventSynchronize(prev);
        held->lock();
        slot.encrypting = false;
        g_slot_cv.notify_all();
        if (!g_s.ready) return nullptr;
    }
    if (slot.owner) harvest(*slot.owner);   // statuses leave the slot before reuse
    if (!ensure_stage(slot, stride * n, layer_ks_stride(count) * n, n, 0, true)) return nullptr;
    if (slot.done) cudaEventSynchronize(slot.done);
    if (slot.hold) {                        // its copy has completed: the buffer goes back to the pool
        std::lock_guard<std::mutex> lock(g_prep.mu);
        prep_release_locked(*slot.hold);
        slot.hold.reset();
    }
    // A pre-encrypted entry for exactly this reload replaces the inline
    // encryption; its tickets were reserved when it was announced.
    std::shared_ptr<Prepared> pre = encrypted ? nullptr : take_prepared(layer, srcs, n, count, codec);

    std::vector<uint64_t> tickets(n);
    if (pre) {
        tickets = pre->tickets;
        g_prep_ready += n;
    } else if (encrypted) {
        if (given_tickets == nullptr) return nullptr;
        for (uint32_t i = 0; i < n; ++i)
            if (!reserve_given_ticket(given_tickets[i])) return nullptr;
        tickets.assign(given_tickets, given_tickets + n);
    } else {
        reserve_tickets(n, tickets.data());
    }
    // The keystream depends only on the tickets: it is generated on the
    // producer stream while the host encrypts and the records cross the link
    // (the slot's previous batch has completed, see above).
    if ((!slot.ks_ready && !CUDA_OK(cudaEventCreateWithFlags(&slot.ks_ready, cudaEventDisableTiming))) ||
        (!slot.copied && !CUDA_OK(cudaEventCreateWithFlags(&slot.copied, cudaEventDisableTiming))))
        return nullptr;
    if (keystream_records_locked(tickets.data(), n, count, slot.ks, g_s.producer) != 0 ||
        !CUDA_OK(cudaEventRecord(slot.ks_ready, g_s.producer)))
        return nullptr;
    const bool ring = !encrypted && !pre && h2d_ring();
    if (pre) {
        for (uint32_t i = 0; i < n; ++i) maybe_tamper_h2d(pre->host + i * stride, count);
    } else if (ring) {
        if (!encrypt_ring_locked(tickets.data(), srcs, n, count, stride, slot.dev)) return nullptr;
    } else if (!encrypted) {
        std::atomic<bool> ok{true};
        uint8_t key[16], salt[4];
        std::memcpy(key, g_s.key, 16);
        std::memcpy(salt, g_s.salt, 4);
        uint8_t* host = slot.host;
        slot.encrypting = true;
        if (held != nullptr) held->unlock();
        pool().parallel_for(n, [&](size_t i) {
            uint8_t iv[16], aad[64];
            iv_for_salt(salt, tickets[i], iv);
            build_aad(srcs[i], count, SECURE_INFER_DIRECTION_H2D, tickets[i], 0, 0, aad);
            if (!encrypt_record(key, iv, aad, static_cast<const uint8_t*>(srcs[i]), count, host + i * stride))
                ok = false;
        });
        OPENSSL_cleanse(key, sizeof(key));
        if (held != nullptr) held->lock();
        slot.encrypting = false;
        g_slot_cv.notify_all();
        if (!ok || !g_s.ready) return nullptr;
        for (uint32_t i = 0; i < n; ++i) maybe_tamper_h2d(slot.host + i * stride, count);
    }

    auto batch = std::make_shared<LayerBatch>();
    batch->layer = layer;
    batch->job = g_s.job;
    batch->n = n;
    batch->count = count;
    if (codec) batch->codec = *codec;
    batch->encrypted = encrypted;
    batch->stream = stream;
    batch->slot = &slot;
    batch->items.resize(n);
    for (uint32_t i = 0; i < n; ++i) batch->items[i] = RetryInfo{encrypted ? nullptr : srcs[i], dsts[i]};
    if (!CUDA_OK(cudaEventCreateWithFlags(&batch->done, cudaEventDisableTiming))) return nullptr;

    // Records cross the link on the copy stream, so the next layer's copy
    // does not queue behind this layer's kernel; the caller's stream waits
    // for the records and the keystream, then runs the fused kernel.
    const void* host_src = encrypted ? srcs[0] : pre ? pre->host : slot.host;
    if ((!ring && !CUDA_OK(cudaMemcpyAsync(slot.dev, host_src, stride * n, cudaMemcpyHostToDevice, g_s.copier))) ||
        !CUDA_OK(cudaEventRecord(slot.copied, g_s.copier)) ||
        !CUDA_OK(cudaStreamWaitEvent(stream, slot.copied, 0)) ||
        !CUDA_OK(cudaStreamWaitEvent(stream, slot.ks_ready, 0)))
        return nullptr;
    if (verify_records_locked(slot.dev, stride, count, n, tickets.data(), dsts, slot.ks, slot.dev_status, codec,
                              stream) != 0)
        return nullptr;
    cudaMemcpyAsync(slot.host_status, slot.dev_status, sizeof(uint32_t) * n, cudaMemcpyDeviceToHost, stream);
    cudaEventRecord(batch->done, stream);
    slot.done = batch->done;
    slot.owner = batch;
    slot.hold = pre;
    return batch;
}

void register_batch_locked(const std::shared_ptr<LayerBatch>& b)
{
    g_s.pending[b->layer].push_back(b);
    std::lock_guard<std::mutex> ev(g_events_mu);
    g_s.last_event[b->layer] = b->done;
    g_s.last_batch[b->layer] = b;
}

// ------------------------------------------------------------ H2D groups
struct Submission {
    void* dst;
    const void* src;
    size_t count;
    cudaStream_t stream;
};

thread_local int t_group_depth = 0;
thread_local std::vector<Submission> t_group;

int flush_submissions(std::vector<Submission>& subs)
{
    // Bucket by (layer, count, stream); each bucket is one staged reload.
    std::map<std::tuple<uint32_t, size_t, cudaStream_t>, std::vector<size_t>> buckets;
    for (size_t i = 0; i < subs.size(); ++i) {
        HostRange r{};
        uint64_t block = 0, off = 0;
        const uint32_t layer = lookup_range(subs[i].src, subs[i].count, &r, &block, &off) ? r.layer : UINT32_MAX;
        buckets[{layer, subs[i].count, subs[i].stream}].push_back(i);
    }
    std::unique_lock<std::recursive_mutex> lock(g_mu);
    for (auto& kv : buckets) {
        std::vector<const void*> srcs;
        std::vector<void*> dsts;
        for (size_t i : kv.second) {
            srcs.push_back(subs[i].src);
            dsts.push_back(subs[i].dst);
        }
        auto b = submit_layer_locked(std::get<0>(kv.first), srcs.data(), dsts.data(), static_cast<uint32_t>(srcs.size()),
                                     std::get<1>(kv.first), nullptr, false, nullptr, std::get<2>(kv.first), &lock);
        if (!b) return -1;
        register_batch_locked(b);
    }
    subs.clear();
    return 0;
}

// ------------------------------------------------------------ D2H
uint64_t g_d2h_batch_id = 0;
thread_local uint64_t t_d2h_batch = 0;
thread_local int t_d2h_group_depth = 0;
thread_local std::vector<Submission> t_d2h_group;

void d2h_worker()
{
    pin_library_thread();
    std::unique_lock<std::mutex> lock(g_d2h_mu);
    for (;;) {
        g_s.d2h_cv.wait(lock, [] { return g_s.d2h_stop || !g_s.d2h_queue.empty(); });
        if (g_s.d2h_queue.empty()) return;
        auto g = g_s.d2h_queue.front();
        g_s.d2h_queue.pop_front();
        lock.unlock();
        cudaEventSynchronize(g->copied);
        const uint64_t stride = record_bytes(g->count), aligned = aligned32(g->count);
        uint64_t nth = g_tamper_d2h_nth.load();
        while (nth != 0 && !g_tamper_d2h_nth.compare_exchange_weak(nth, nth > g->n ? nth - g->n : 0)) {}
        if (nth != 0 && nth <= g->n) g->slot->host[(nth - 1) * stride] ^= 0x01;   // secure_infer.cpp:2454-2468
        std::atomic<bool> ok{true};
        const uint8_t* key = g_s.key;
        pool().parallel_for(g->n, [&](size_t i) {
            const uint8_t* rec = g->slot->host + i * stride;
            if (!decrypt_record(key, &g->ivs[16 * i], &g->aads[64 * i], rec, g->count, rec + aligned,
                                static_cast<uint8_t*>(g->dsts[i])))
                ok = false;
        });
        lock.lock();
        g->ok = ok.load();
        g->verified = true;
        if (g->ok) g_verified += g->n; else g_rejected += g->n;
        g_s.d2h_cv.notify_all();
    }
}

// Device half of a writeback of n blocks (transport_codec.py:22-42 encode,
// ghash.aicpu:656-699 encrypt_tag): for codec blocks quantise into packets,
// then keystream + tag masks, then the fused encrypt/GHASH/tag kernel writing
// records C || tag || 0^16 || AAD into `records` (device, `stride` apart).
// Each record gets a fresh ticket; its AAD names host_dsts[i] with direction
// D2H (secure_infer.cpp:730-775).  tickets/ivs/aads (host, optional) receive
// what the host verify needs.  `slot` must hold n records of scratch.
// Caller holds g_mu.
int writeback_device_locked(const void* const* srcs, void* const* host_dsts, uint32_t n, const CodecParams& cp,
                            uint32_t codec_layer, uint64_t count, uint8_t* records, uint64_t stride, StageSlot& slot,
                            uint64_t* tickets, uint8_t* ivs, uint8_t* aads, cudaStream_t stream)
{
    const uint64_t ks_stride = layer_ks_stride(count);
    std::vector<uint64_t> tk(n);
    bool unaligned = misaligned(records) || (stride & 15u);
    reserve_tickets(n, tk.data());
    for (uint32_t i = 0; i < n; ++i) {
        if (tickets) tickets[i] = tk[i];
        if (ivs) iv_for(tk[i], ivs + 16ull * i);
        build_aad(host_dsts ? host_dsts[i] : nullptr, count, SECURE_INFER_DIRECTION_D2H, tk[i], 0, 0,
                  slot.host_aad + 64ull * i);
        if (aads) std::memcpy(aads + 64ull * i, slot.host_aad + 64ull * i, 64);
        slot.host_ptrs[i] = static_cast<const uint8_t*>(srcs[i]);
        if (!cp.bits && misaligned(srcs[i])) unaligned = true;
    }
    if (!CUDA_OK(cudaMemcpyAsync(slot.dev_aad, slot.host_aad, 64ull * n, cudaMemcpyHostToDevice, stream))) return -1;
    const uint32_t v_first = cp.kind == SECURE_INFER_KIND_KV ? n / 2 : (cp.kind == 1 ? 0u : n);
    // The keystream needs only the tickets: it runs on the producer stream
    // beside the quantiser (the two kernels share SMs: one is bound by the
    // shared-memory pipe, the other by issue), and the encrypt kernel waits
    // for both.  The producer first waits for this stream's earlier work, the
    // slot's previous user.
    if ((!slot.ks_ready && !CUDA_OK(cudaEventCreateWithFlags(&slot.ks_ready, cudaEventDisableTiming))) ||
        (!slot.copied && !CUDA_OK(cudaEventCreateWithFlags(&slot.copied, cudaEventDisableTiming))))
        return -1;
    if (!CUDA_OK(cudaEventRecord(slot.copied, stream)) || !CUDA_OK(cudaStreamWaitEvent(g_s.producer, slot.copied, 0)))
        return -1;
    if (keystream_records_locked(tk.data(), n, count, slot.ks, g_s.producer) != 0 ||
        !CUDA_OK(cudaEventRecord(slot.ks_ready, g_s.producer)))
        return -1;
    if (cp.bits) {
        if (!CUDA_OK(cudaMemcpyAsync(slot.dev_ptrs, slot.host_ptrs, sizeof(void*) * n, cudaMemcpyHostToDevice, stream)))
            return -1;
        EncodeLaunch E{};
        E.srcs = slot.dev_ptrs;
        E.packets = slot.pkt;
        E.n = n;
        E.width = static_cast<uint32_t>(count);
        E.layer = codec_layer;
        E.codec = cp;
        E.v_first = v_first;
        if (launch_encode(E, stream) != cudaSuccess) return -1;
    }
    if (!CUDA_OK(cudaStreamWaitEvent(stream, slot.ks_ready, 0))) return -1;
    std::vector<LayerRec> recs(std::min<uint32_t>(n, kLayerCapLarge));
    for (uint32_t first = 0; first < n; first += kLayerCapLarge) {
        const uint32_t m = std::min<uint32_t>(n - first, kLayerCapLarge);
        uint32_t seg_steps = 0, nseg = 0;
        layer_segments_for(count, m, 0, &seg_steps, &nseg);
        LaunchSlot& ls = g_s.launch[g_s.launch_next];
        g_s.launch_next = (g_s.launch_next + 1) % g_s.launch.size();
        if (!ensure_launch_slot(ls, m, nseg * m)) return -1;
        LayerHeader h{};
        std::memcpy(h.rk, g_s.rk, sizeof(h.rk));
        h.sched = g_s.sched;
        h.records = records + first * stride;
        h.stride = stride;
        h.count = count;
        h.ks = slot.ks + first * ks_stride;
        h.ks_stride = ks_stride;
        h.status = slot.dev_status + first;
        h.partials = ls.partials;
        h.counters = ls.counters;
        h.iv0 = load_be32(g_s.salt);
        h.n = m;
        h.nseg = nseg;
        h.seg_steps = seg_steps;
        h.join_pow = sib::join_tables_for(g_s.join_tabs, seg_steps);
        h.aad = slot.dev_aad + 64ull * first;
        h.unaligned = unaligned ? 1u : 0u;
        for (uint32_t i = 0; i < m; ++i) {
            uint8_t* plain = cp.bits ? slot.pkt + (first + i) * count : const_cast<uint8_t*>(slot.host_ptrs[first + i]);
            recs[i] = LayerRec{plain, tk[first + i]};
        }
        if (launch_layer_encrypt(h, recs.data(), stream) != cudaSuccess) return -1;
        cudaEventRecord(ls.free_ev, stream);
        ls.used = true;
    }
    return 0;
}

int d2h_submit_group(const void* const* srcs, void* const* dsts, uint32_t n, uint64_t count,
                     const secure_infer_codec* codec, cudaStream_t stream)
{
    CodecParams cp;
    uint64_t packet = 0;
    if (!codec_geometry(codec, &cp, &packet, true) || n == 0 || srcs == nullptr || dsts == nullptr) return -1;
    if (cp.bits) count = packet;
    if (count == 0 || (cp.bits && cp.kind == SECURE_INFER_KIND_KV && (n & 1u))) return -1;
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!g_s.ready) return -1;
    const uint64_t stride = record_bytes(count);
    StageSlot& slot = g_s.d2h[g_s.d2h_next];
    g_s.d2h_next = (g_s.d2h_next + 1) % g_s.d2h.size();
    {
        // The slot's previous group must be verified before its host copy is reused.
        std::unique_lock<std::mutex> dl(g_d2h_mu);
        g_s.d2h_cv.wait(dl, [&] {
            for (auto& g : g_s.d2h_all)
                if (g->slot == &slot && !g->verified) return false;
            return true;
        });
    }
    if (!ensure_stage(slot, stride * n, layer_ks_stride(count) * n, n, cp.bits ? packet * n : 0)) return -1;
    auto g = std::make_shared<D2HGroup>();
    g->n = n;
    g->count = count;
    g->slot = &slot;
    g->batch = t_d2h_batch;
    g->dsts.assign(dsts, dsts + n);
    g->ivs.resize(16ull * n);
    g->aads.resize(64ull * n);
    if (!CUDA_OK(cudaEventCreateWithFlags(&g->copied, cudaEventDisableTiming))) return -1;
    if (writeback_device_locked(srcs, dsts, n, cp, codec ? codec->layer : 0, count, slot.dev, stride, slot, nullptr,
                                g->ivs.data(), g->aads.data(), stream) != 0)
        return -1;
    if (!CUDA_OK(cudaMemcpyAsync(slot.host, slot.dev, stride * n, cudaMemcpyDeviceToHost, stream))) return -1;
    cudaEventRecord(g->copied, stream);
    {
        std::lock_guard<std::mutex> dl(g_d2h_mu);
        g_s.d2h_queue.push_back(g);
        g_s.d2h_all.push_back(g);
    }
    g_s.d2h_cv.notify_all();
    return 0;
}

// Waits for D2H groups of `batch` (0 = all); drops finished groups.
int d2h_join(uint64_t batch, bool device_only)
{
    std::unique_lock<std::mutex> dl(g_d2h_mu);
    if (device_only) {
        std::vector<cudaEvent_t> evs;
        for (auto& g : g_s.d2h_all)
            if (batch == 0 || g->batch == batch) evs.push_back(g->copied);
        dl.unlock();
        for (auto e : evs) cudaEventSynchronize(e);
        return 0;
    }
    g_s.d2h_cv.wait(dl, [&] {
        for (auto& g : g_s.d2h_all)
            if ((batch == 0 || g->batch == batch) && !g->verified) return false;
        return true;
    });
    bool ok = true;
    for (auto it = g_s.d2h_all.begin(); it != g_s.d2h_all.end();) {
        if (batch == 0 || (*it)->batch == batch) {
            ok = ok && (*it)->ok;
            cudaEventDestroy((*it)->copied);
            it = g_s.d2h_all.erase(it);
        } else {
            ++it;
        }
    }
    return ok ? 0 : -1;
}

int d2h_flush_thread_group()
{
    std::map<std::pair<size_t, cudaStream_t>, std::vector<size_t>> buckets;
    for (size_t i = 0; i < t_d2h_group.size(); ++i)
        buckets[{t_d2h_group[i].count, t_d2h_group[i].stream}].push_back(i);
    for (auto& kv : buckets) {
        std::vector<const void*> srcs;
        std::vector<void*> dsts;
        for (size_t i : kv.second) {
            srcs.push_back(t_d2h_group[i].src);
            dsts.push_back(t_d2h_group[i].dst);
        }
        if (d2h_submit_group(srcs.data(), dsts.data(), static_cast<uint32_t>(srcs.size()), kv.first.first, nullptr,
                             kv.first.second) != 0)
            return -1;
    }
    t_d2h_group.clear();
    return 0;
}

void shutdown_locked()
{
    host_only_session = false;
    if (!g_s.ready) return;
    cudaDeviceSynchronize();
    prep_shutdown();
    {
        std::lock_guard<std::mutex> dl(g_d2h_mu);
        g_s.d2h_stop = true;
    }
    g_s.d2h_cv.notify_all();
    if (g_s.d2h_thread.joinable()) g_s.d2h_thread.join();
    for (auto& g : g_s.d2h_all) cudaEventDestroy(g->copied);
    g_s.d2h_all.clear();
    g_s.d2h_queue.clear();
    for (auto& kv : g_s.pending)
        for (auto& b : kv.second) harvest(*b);
    g_s.pending.clear();
    {
        std::lock_guard<std::mutex> ev(g_events_mu);
        g_s.last_event.clear();
        g_s.last_batch.clear();
    }
    for (auto& s : g_s.h2d) {
        s.owner.reset();
        free_stage(s);
        if (s.ks_ready) cudaEventDestroy(s.ks_ready);
        if (s.copied) cudaEventDestroy(s.copied);
        s.ks_ready = s.copied = nullptr;
    }
    for (auto& s : g_s.d2h) {
        free_stage(s);
        if (s.ks_ready) cudaEventDestroy(s.ks_ready);
        if (s.copied) cudaEventDestroy(s.copied);
        s.ks_ready = s.copied = nullptr;
    }
    for (auto& s : g_s.wb) {
        free_stage(s);
        if (s.done) cudaEventDestroy(s.done);
        if (s.ks_ready) cudaEventDestroy(s.ks_ready);
        if (s.copied) cudaEventDestroy(s.copied);
        s.done = s.ks_ready = s.copied = nullptr;
    }
    for (auto& s : g_s.launch) {
        cudaFreeHost(s.host_recs); cudaFreeHost(s.host_jobs);
        cudaFree(s.dev_recs); cudaFree(s.dev_jobs); cudaFree(s.partials); cudaFree(s.counters);
        if (s.free_ev) cudaEventDestroy(s.free_ev);
    }
    g_s.launch.clear();
    g_s.h2d.clear();
    for (auto& rc : g_s.ring) {
        if (rc.ev) cudaEventSynchronize(rc.ev);
        if (rc.host) cudaFreeHost(rc.host);
        if (rc.ev) cudaEventDestroy(rc.ev);
    }
    g_s.ring.clear();
    g_s.ring_next = 0;
    g_s.d2h.clear();
    g_s.wb.clear();
    cudaFree(g_s.sched);
    g_s.sched = nullptr;
    cudaFree(g_s.join_tabs);
    g_s.join_tabs = nullptr;
    if (g_s.producer) cudaStreamDestroy(g_s.producer);
    g_s.producer = nullptr;
    if (g_s.copier) cudaStreamDestroy(g_s.copier);
    g_s.copier = nullptr;
    if (g_s.consumed_ev) cudaEventDestroy(g_s.consumed_ev);
    if (g_s.produced_ev) cudaEventDestroy(g_s.produced_ev);
    g_s.consumed_ev = g_s.produced_ev = nullptr;
    OPENSSL_cleanse(g_s.key, sizeof(g_s.key));
    OPENSSL_cleanse(g_s.rk, sizeof(g_s.rk));
    g_s.ready = false;
}

}  // namespace
}  // namespace host
}  // namespace sib

using namespace sib::host;
using sib::launch_schedule;

#define SI_EXPORT extern "C" __attribute__((visibility("default")))

namespace {
// Session setup shared by the two entry points.  device_key: the key already
// in device memory (key agreement), or null to copy key16 to the device.
int session_init_locked(int device, const uint8_t* key16, const uint8_t* iv_salt4, const void* device_key);
}  // namespace

// ------------------------------------------------ asynchronous layer loop
// secure_infer_h2d_reload_layers_async: the connector's per-layer fetch loop
// (reuse/connector.py:222-331) run by a library thread, so the reloads of a
// request never wait for the Python interpreter while the model thread
// launches attention.  One request at a time.
namespace {
struct AsyncReload {
    uint32_t first = 0, nlayers = 0, n = 0;
    std::vector<const void*> srcs;          // [nlayers][n]
    std::vector<void*> dsts;                // [nlayers][n]
    std::vector<uint64_t> counts;           // [nlayers]
    std::vector<secure_infer_codec> codecs; // [nlayers], bits 0 = raw
    bool lookahead = true;
    cudaStream_t stream = nullptr;
    std::vector<uint8_t> state;             // per layer: 0 pending, 1 submitted, 2 failed
    int rc = 0;
    std::thread worker;

    // A request that was never joined (process exit) lets its thread go; the
    // last owner may be that thread itself.
    ~AsyncReload()
    {
        if (worker.joinable()) worker.detach();
    }
};
std::mutex g_async_mu;
std::condition_variable g_async_cv;
std::shared_ptr<AsyncReload> g_async;

}  // namespace

extern "C" int secure_infer_h2d_reload_layer(uint32_t, const void* const*, void* const*, uint32_t, uint64_t,
                                             const secure_infer_codec*, int, const uint64_t*, void*);
extern "C" int secure_infer_h2d_prepare_layer(uint32_t, const void* const*, uint32_t, uint64_t,
                                              const secure_infer_codec*);
extern "C" void secure_infer_retire_transfer_prefetches(void);

namespace {
void async_worker(std::shared_ptr<AsyncReload> a)
{
    pin_library_thread();
    const uint32_t n = a->n;
    for (uint32_t i = 0; i < a->nlayers; ++i) {
        // Announce the next layer first (pre-encryption lookahead); a refused
        // announcement only means that layer is encrypted inline.
        if (a->lookahead && i + 1 < a->nlayers)
            secure_infer_h2d_prepare_layer(a->first + i + 1, &a->srcs[(i + 1ull) * n], n, a->counts[i + 1],
                                           &a->codecs[i + 1]);
        const int rc = secure_infer_h2d_reload_layer(a->first + i, &a->srcs[1ull * i * n], &a->dsts[1ull * i * n], n,
                                                     a->counts[i], &a->codecs[i], 0, nullptr, a->stream);
        {
            std::lock_guard<std::mutex> lock(g_async_mu);
            if (rc != 0) {
                a->rc = -1;
                for (uint32_t j = i; j < a->nlayers; ++j) a->state[j] = 2;
            } else {
                a->state[i] = 1;
            }
        }
        g_async_cv.notify_all();
        if (rc != 0) break;
    }
    if (a->lookahead) secure_infer_retire_transfer_prefetches();
}

// Waits until `layer` of the active asynchronous request (when it covers that
// layer) has been submitted; false if its submission failed or the worker
// gave no answer within two minutes.
bool await_async_layer(uint32_t layer)
{
    std::unique_lock<std::mutex> lock(g_async_mu);
    const std::shared_ptr<AsyncReload> a = g_async;
    if (!a || layer < a->first || layer - a->first >= a->nlayers) return true;
    const uint32_t i = layer - a->first;
    if (!g_async_cv.wait_for(lock, std::chrono::seconds(120), [&] { return a->state[i] != 0; })) return false;
    return a->state[i] == 1;
}

// A session change waits for submissions that are encrypting into staging
// slots with the session lock released (they take it back to finish).
void wait_encrypting(std::unique_lock<std::recursive_mutex>& lock)
{
    g_slot_cv.wait(lock, [] {
        for (const auto& slot : g_s.h2d)
            if (slot.encrypting) return false;
        return true;
    });
}

// Joins the active request's worker; its result (0, or -1 if a reload failed).
int join_async()
{
    std::shared_ptr<AsyncReload> a;
    {
        std::lock_guard<std::mutex> lock(g_async_mu);
        a = g_async;
    }
    if (!a) return 0;
    if (a->worker.joinable()) a->worker.join();
    std::lock_guard<std::mutex> lock(g_async_mu);
    if (g_async == a) g_async.reset();
    return a->rc;
}
}  // namespace

SI_EXPORT int secure_infer_h2d_reload_layers_async(uint32_t first_layer, uint32_t nlayers, const void* const* srcs,
                                                   void* const* dsts, uint32_t n, const uint64_t* counts,
                                                   const secure_infer_codec* codecs, int lookahead, void* stream)
{
    if (srcs == nullptr || dsts == nullptr || counts == nullptr || nlayers == 0 || n == 0) return -1;
    if (UINT32_MAX - first_layer < nlayers) return -1;
    join_async();   // one request at a time
    auto a = std::make_shared<AsyncReload>();
    a->first = first_layer;
    a->nlayers = nlayers;
    a->n = n;
    a->srcs.assign(srcs, srcs + 1ull * nlayers * n);
    a->dsts.assign(dsts, dsts + 1ull * nlayers * n);
    a->counts.assign(counts, counts + nlayers);
    a->codecs.assign(nlayers, secure_infer_codec{});
    if (codecs != nullptr) a->codecs.assign(codecs, codecs + nlayers);
    a->lookahead = lookahead != 0;
    a->stream = static_cast<cudaStream_t>(stream);
    a->state.assign(nlayers, 0);
    {
        std::lock_guard<std::mutex> lock(g_async_mu);
        g_async = a;
    }
    a->worker = std::thread(async_worker, a);
    return 0;
}

SI_EXPORT int secure_infer_h2d_reload_layers_join(void) { return join_async(); }

SI_EXPORT int secure_infer_session_init(int device, const uint8_t* key16, const uint8_t* iv_salt4)
{
    if (key16 == nullptr || iv_salt4 == nullptr) return -1;
    join_async();   // a running layer loop finishes under the old session
    std::unique_lock<std::recursive_mutex> lock(g_mu);
    wait_encrypting(lock);
    return session_init_locked(device, key16, iv_salt4, nullptr);
}

SI_EXPORT int secure_infer_session_init_key_agreement(int device)
{
    if (device < 0) return -1;
    join_async();
    std::unique_lock<std::recursive_mutex> lock(g_mu);
    wait_encrypting(lock);
    shutdown_locked();
    if (!CUDA_OK(cudaSetDevice(device))) return -1;
    // Host half (secure_infer.cpp:449-521): fresh X25519 secret and challenge.
    uint8_t secret[32], challenge[32], host_public[32], device_public[32], proof[32], shared[32];
    uint8_t key[16], expected[32], salt[4];
    int32_t status = -1;
    if (RAND_bytes(secret, sizeof(secret)) != 1 || RAND_bytes(challenge, sizeof(challenge)) != 1) return -1;
    kx::x25519_public(host_public, secret);
    uint8_t* d = nullptr;   // [0,32) host public, [32,64) challenge, [64,96) device public, [96,128) proof,
                            // [128,144) key, [160,164) status
    cudaStream_t setup = nullptr;
    bool ok = CUDA_OK(cudaMalloc(&d, 192)) && CUDA_OK(cudaStreamCreateWithFlags(&setup, cudaStreamNonBlocking)) &&
              CUDA_OK(cudaMemcpyAsync(d, host_public, 32, cudaMemcpyHostToDevice, setup)) &&
              CUDA_OK(cudaMemcpyAsync(d + 32, challenge, 32, cudaMemcpyHostToDevice, setup)) &&
              sib::launch_key_agreement(d, d + 32, d + 128, d + 64, d + 96, reinterpret_cast<int32_t*>(d + 160),
                                        setup) == cudaSuccess &&
              CUDA_OK(cudaMemcpyAsync(device_public, d + 64, 32, cudaMemcpyDeviceToHost, setup)) &&
              CUDA_OK(cudaMemcpyAsync(proof, d + 96, 32, cudaMemcpyDeviceToHost, setup)) &&
              CUDA_OK(cudaMemcpyAsync(&status, d + 160, 4, cudaMemcpyDeviceToHost, setup)) &&
              CUDA_OK(cudaStreamSynchronize(setup)) && status == 0;
    if (ok) {
        kx::x25519(shared, secret, device_public);
        uint8_t nonzero = 0;
        for (uint8_t b : shared) nonzero |= b;
        kx::derive_key(key, shared, host_public, device_public, challenge);
        kx::derive_proof(expected, key, challenge);
        kx::derive_salt(salt, shared);
        uint8_t diff = 0;
        for (int i = 0; i < 32; ++i) diff |= static_cast<uint8_t>(expected[i] ^ proof[i]);
        ok = nonzero != 0 && diff == 0;
    }
    // The device builds its schedule from its own copy of the key, which then
    // is wiped with the rest of the handshake buffer.
    if (ok) ok = session_init_locked(device, key, salt, d + 128) == 0;
    if (d) {
        cudaMemset(d, 0, 192);
        cudaDeviceSynchronize();
        cudaFree(d);
    }
    if (setup) cudaStreamDestroy(setup);
    OPENSSL_cleanse(secret, sizeof(secret));
    OPENSSL_cleanse(shared, sizeof(shared));
    OPENSSL_cleanse(key, sizeof(key));
    OPENSSL_cleanse(salt, sizeof(salt));
    return ok ? 0 : -1;
}

namespace {
// The keystream producer runs at the device's highest stream priority: a
// reload's kernels gate the attention that waits for its layer, so their CTAs
// are scheduled ahead of compute work queued on normal-priority streams.
cudaError_t create_priority_stream(cudaStream_t* s)
{
    int least = 0, greatest = 0;
    if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) greatest = 0;
    return cudaStreamCreateWithPriority(s, cudaStreamNonBlocking, greatest);
}

int session_init_locked(int device, const uint8_t* key16, const uint8_t* iv_salt4, const void* device_key)
{
    shutdown_locked();
    host_only_session = false;
    g_s.device = device;
    std::memcpy(g_s.key, key16, 16);
    std::memcpy(g_s.salt, iv_salt4, 4);
    g_key_generation.fetch_add(1, std::memory_order_acq_rel);   // re-key the host OpenSSL contexts
    {
        std::lock_guard<std::mutex> rl(g_s.replay_mu);
        g_s.outstanding.clear();
    }
    g_s.job = 0;
    if (device < 0) {
        // Host-only session: record encryption, tickets and AAD work without
        // a GPU; every device entry point still reports failure.
        host_only_session = true;
        return 0;
    }
    if (!CUDA_OK(cudaSetDevice(device))) return -1;
    uint8_t* dkey = nullptr;
    if (!CUDA_OK(cudaMalloc(&g_s.sched, sib::schedule_bytes())) ||
        !CUDA_OK(cudaMemset(g_s.sched, 0, sib::schedule_bytes())) ||
        !CUDA_OK(cudaMalloc(&g_s.join_tabs, sib::join_tables_bytes())) || !CUDA_OK(cudaMalloc(&dkey, 16)) ||
        !CUDA_OK(device_key ? cudaMemcpy(dkey, device_key, 16, cudaMemcpyDeviceToDevice)
                            : cudaMemcpy(dkey, key16, 16, cudaMemcpyHostToDevice)) ||
        !CUDA_OK(create_priority_stream(&g_s.producer)) ||
        !CUDA_OK(cudaStreamCreateWithFlags(&g_s.copier, cudaStreamNonBlocking)) ||
        !CUDA_OK(cudaEventCreateWithFlags(&g_s.consumed_ev, cudaEventDisableTiming)) ||
        !CUDA_OK(cudaEventCreateWithFlags(&g_s.produced_ev, cudaEventDisableTiming))) {
        cudaFree(dkey);
        return -1;
    }
    // H = E_K(0^128) and the GHASH tables are derived on the device; the key
    // copy used for the derivation is wiped and freed right after.
    const bool ok = launch_schedule(g_s.sched, dkey, nullptr, true, g_s.producer) == cudaSuccess &&
                    CUDA_OK(cudaMemsetAsync(dkey, 0, 16, g_s.producer)) &&
                    sib::launch_join_tables(g_s.sched, g_s.join_tabs, g_s.producer) == cudaSuccess &&
                    CUDA_OK(cudaStreamSynchronize(g_s.producer)) &&
                    CUDA_OK(cudaMemcpy(g_s.rk, g_s.sched, sizeof(g_s.rk), cudaMemcpyDeviceToHost));   // rk leads the schedule
    cudaFree(dkey);
    if (!ok) return -1;
    g_s.launch.resize(kLaunchSlots);
    for (auto& s : g_s.launch) cudaEventCreateWithFlags(&s.free_ev, cudaEventDisableTiming);
    g_s.h2d.resize(stage_slot_count());
    g_s.wb.resize(stage_slot_count());
    g_s.d2h.resize(stage_slot_count());
    g_s.d2h_stop = false;
    g_s.d2h_thread = std::thread(d2h_worker);
    g_verified = g_rejected = g_retried = 0;
    g_s.ready = true;
    return 0;
}
}  // namespace

SI_EXPORT int secure_infer_session_shutdown(void)
{
    join_async();   // outside the session lock: the worker takes it per layer
    std::unique_lock<std::recursive_mutex> lock(g_mu);
    wait_encrypting(lock);
    shutdown_locked();
    return 0;
}

SI_EXPORT void secure_infer_register_host_range_ex(const void* base, size_t bytes, uint32_t layer_id,
                                                   uint32_t tensor_kind, size_t block_bytes)
{
    if (base == nullptr || bytes == 0) return;
    const uintptr_t b = reinterpret_cast<uintptr_t>(base);
    if (bytes > UINTPTR_MAX - b) return;
    std::unique_lock<std::shared_mutex> lock(g_ranges_mu);
    // The new registration is the newest; older ones it covers completely can
    // never match again and are dropped, so re-registering a recycled buffer
    // does not grow the list.
    g_ranges.erase(std::remove_if(g_ranges.begin(), g_ranges.end(),
                                  [&](const HostRange& r) { return r.begin >= b && r.end <= b + bytes; }),
                   g_ranges.end());
    g_ranges.push_back({b, b + bytes, layer_id, tensor_kind, block_bytes});
}

SI_EXPORT void secure_infer_register_host_range(const void* base, size_t bytes)
{
    secure_infer_register_host_range_ex(base, bytes, UINT32_MAX, UINT32_MAX, 0);
}

SI_EXPORT int secure_infer_host_pool_info(uint32_t* threads, int32_t* cpus, uint32_t max_cpus, uint32_t* pinned)
{
    if (threads == nullptr) return -1;
    const PoolPlan& plan = pool_plan();
    *threads = static_cast<uint32_t>(pool().size());
    if (pinned) *pinned = plan.pinned ? 1u : 0u;
    for (uint32_t i = 0; cpus != nullptr && i < max_cpus && i < plan.cpus.size(); ++i) cpus[i] = plan.cpus[i];
    return static_cast<int>(plan.cpus.size());
}

SI_EXPORT int secure_infer_is_registered_host_range(const void* ptr, size_t bytes)
{
    if (ptr == nullptr || bytes == 0) return 0;
    HostRange r{};
    uint64_t block = 0, off = 0;
    return lookup_range(ptr, bytes, &r, &block, &off) ? 1 : 0;
}

SI_EXPORT uint64_t secure_infer_new_transfer_ticket(void)
{
    uint64_t t = 0;
    issue_tickets(1, &t);
    return t;
}

SI_EXPORT int secure_infer_derive_transfer_iv(const uint8_t* base_iv16, uint64_t ticket, uint64_t block_offset,
                                              uint8_t* out_iv16)
{
    if (base_iv16 == nullptr || out_iv16 == nullptr || ticket == 0 || block_offset > UINT32_MAX - 2u) return -1;
    std::memcpy(out_iv16, base_iv16, 16);
    store_be64(out_iv16 + 4, ticket);
    store_be32(out_iv16 + 12, static_cast<uint32_t>(block_offset + 2u));
    return 0;
}

SI_EXPORT int secure_infer_build_gcm_aad(const void* host_ptr, size_t bytes, uint8_t direction, uint64_t ticket,
                                         uint64_t transfer_offset, uint8_t* out64)
{
    if (out64 == nullptr || host_ptr == nullptr || bytes == 0 || ticket == 0 ||
        (direction != SECURE_INFER_DIRECTION_H2D && direction != SECURE_INFER_DIRECTION_D2H))
        return -1;
    build_aad(host_ptr, bytes, direction, ticket, transfer_offset, 0, out64);
    return 0;
}

SI_EXPORT uint64_t secure_infer_record_bytes(uint64_t count) { return record_bytes(count); }

SI_EXPORT int secure_infer_h2d_encrypt_records(const void* const* srcs, uint64_t count, uint32_t n, void* records,
                                               uint64_t record_stride, uint64_t* tickets_out)
{
    if (srcs == nullptr || records == nullptr || n == 0 || count == 0 || record_stride < record_bytes(count))
        return -1;
    std::vector<uint64_t> tickets(n);
    uint8_t key[16];
    {
        std::lock_guard<std::recursive_mutex> lock(g_mu);
        if (!g_s.ready && !host_only_session) return -1;
        std::memcpy(key, g_s.key, 16);
        issue_tickets(n, tickets.data());
    }
    std::atomic<bool> ok{true};
    uint8_t* out = static_cast<uint8_t*>(records);
    pool().parallel_for(n, [&](size_t i) {
        uint8_t iv[16], aad[64];
        iv_for(tickets[i], iv);
        build_aad(srcs[i], count, SECURE_INFER_DIRECTION_H2D, tickets[i], 0, 0, aad);
        if (!encrypt_record(key, iv, aad, static_cast<const uint8_t*>(srcs[i]), count, out + i * record_stride))
            ok = false;
    });
    if (tickets_out) std::memcpy(tickets_out, tickets.data(), sizeof(uint64_t) * n);
    return ok ? 0 : -1;
}

SI_EXPORT uint64_t secure_infer_codec_packet_bytes(uint32_t heads, uint32_t bits)
{
    secure_infer_codec c{bits, 0, heads, 0};
    sib::CodecParams cp;
    uint64_t packet = 0;
    if (bits == 0 || !codec_geometry(&c, &cp, &packet)) return 0;
    return packet;
}

SI_EXPORT int secure_infer_reload_records(uint32_t layer, const void* records, uint64_t record_stride, uint64_t count,
                                          uint32_t n, const uint64_t* tickets, void* const* dsts, void* keystream,
                                          uint32_t* status, const secure_infer_codec* codec, void* stream,
                                          void* producer_stream)
{
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    return reload_records_locked(layer, static_cast<const uint8_t*>(records), record_stride, count, n, tickets, dsts,
                                 static_cast<uint8_t*>(keystream), status, codec, static_cast<cudaStream_t>(stream),
                                 producer_stream ? static_cast<cudaStream_t>(producer_stream) : g_s.producer);
}

SI_EXPORT int secure_infer_keystream_records(const uint64_t* tickets, uint32_t n, uint64_t count, void* keystream,
                                             void* stream)
{
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    return keystream_records_locked(tickets, n, count, static_cast<uint8_t*>(keystream),
                                    static_cast<cudaStream_t>(stream));
}

SI_EXPORT int secure_infer_verify_records(uint32_t layer, const void* records, uint64_t record_stride, uint64_t count,
                                          uint32_t n, const uint64_t* tickets, void* const* dsts,
                                          const void* keystream, uint32_t* status, const secure_infer_codec* codec,
                                          void* stream)
{
    (void)layer;
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    return verify_records_locked(static_cast<const uint8_t*>(records), record_stride, count, n, tickets, dsts,
                                 static_cast<const uint8_t*>(keystream), status, codec,
                                 static_cast<cudaStream_t>(stream));
}

SI_EXPORT int secure_infer_h2d_reload_layer(uint32_t layer, const void* const* srcs, void* const* dsts, uint32_t n,
                                            uint64_t count, const secure_infer_codec* codec,
                                            int records_are_encrypted, const uint64_t* tickets, void* stream)
{
    std::unique_lock<std::recursive_mutex> lock(g_mu);
    auto b = submit_layer_locked(layer, srcs, dsts, n, count, codec, records_are_encrypted != 0, tickets,
                                 static_cast<cudaStream_t>(stream), &lock);
    if (!b) return -1;
    register_batch_locked(b);
    return 0;
}

SI_EXPORT int secure_infer_h2d_prepare_layer(uint32_t layer, const void* const* srcs, uint32_t n, uint64_t count,
                                             const secure_infer_codec* codec)
{
    if (srcs == nullptr || n == 0 || count == 0) return -1;
    for (uint32_t i = 0; i < n; ++i)
        if (srcs[i] == nullptr) return -1;
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!g_s.ready) return -1;
    sib::CodecParams cp;
    uint64_t packet = 0;
    if (!codec_geometry(codec, &cp, &packet, true)) return -1;
    if (cp.bits && (count != packet || (cp.kind == SECURE_INFER_KIND_KV && (n & 1u)))) return -1;
    auto e = std::make_shared<Prepared>();
    e->layer = layer;
    e->srcs.assign(srcs, srcs + n);
    e->count = count;
    e->stride = record_bytes(count);
    e->generation = g_generation.load();
    if (codec) {
        e->has_codec = true;
        e->codec = *codec;
    }
    {
        std::lock_guard<std::mutex> pl(g_prep.mu);
        for (const auto& x : g_prep.entries)   // the same announcement is already pending
            if (x->layer == layer && x->count == count && x->generation == e->generation && x->srcs == e->srcs &&
                same_codec(*x, codec))
                return 1;
        uint64_t got = 0;
        e->host = prep_buffer_locked(e->stride * n, &got);
        if (e->host == nullptr) return 1;
        e->bytes = got;
    }
    std::memcpy(e->key, g_s.key, 16);
    e->tickets.resize(n);
    e->ivs.resize(16ull * n);
    e->aads.resize(64ull * n);
    reserve_tickets(n, e->tickets.data());
    for (uint32_t i = 0; i < n; ++i) {
        iv_for(e->tickets[i], &e->ivs[16ull * i]);
        build_aad(srcs[i], count, SECURE_INFER_DIRECTION_H2D, e->tickets[i], 0, 0, &e->aads[64ull * i]);
    }
    {
        std::lock_guard<std::mutex> pl(g_prep.mu);
        if (!g_prep.worker.joinable()) {
            g_prep.stop = false;
            g_prep.worker = std::thread(prep_worker);
        }
        g_prep.entries.push_back(e);
        g_prep.queue.push_back(e);
    }
    g_prep.cv.notify_all();
    return 0;
}

SI_EXPORT int secure_infer_layer_ready_wait(uint32_t layer, void* stream)
{
    if (!await_async_layer(layer)) return -1;
    // Not the session lock: a submission may hold that across its GPU waits.
    std::lock_guard<std::mutex> lock(g_events_mu);
    auto it = g_s.last_event.find(layer);
    if (it == g_s.last_event.end()) return -1;
    return CUDA_OK(cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), it->second, 0)) ? 0 : -1;
}

SI_EXPORT int secure_infer_h2d_layer_group_begin(size_t expected_tasks)
{
    if (t_group_depth++ == 0) {
        t_group.clear();
        t_group.reserve(expected_tasks);
    }
    return 0;
}

SI_EXPORT int secure_infer_h2d_layer_group_end(void)
{
    if (t_group_depth == 0) return -1;
    if (--t_group_depth != 0) return 0;
    return flush_submissions(t_group);
}

SI_EXPORT int secure_infer_h2d_submit(void* dst, size_t dst_capacity, const void* src, size_t count, void* stream)
{
    if (dst == nullptr || src == nullptr || count == 0 || dst_capacity < count) return -1;
    if (t_group_depth > 0) {
        t_group.push_back({dst, src, count, static_cast<cudaStream_t>(stream)});
        return 0;
    }
    std::vector<Submission> one{{dst, src, count, static_cast<cudaStream_t>(stream)}};
    return flush_submissions(one);
}

SI_EXPORT int secure_infer_recovery_wait_layer_authentication(uint32_t layer)
{
    if (!await_async_layer(layer)) return -1;
    std::vector<std::shared_ptr<LayerBatch>> batches;
    {
        std::lock_guard<std::recursive_mutex> lock(g_mu);
        auto it = g_s.pending.find(layer);
        if (it == g_s.pending.end()) return 0;
        batches.swap(it->second);
        g_s.pending.erase(it);
    }
    bool ok = true;
    for (auto& b : batches) {
        // Wait for the batch without the session lock, so other threads keep
        // submitting meanwhile (the batch owns its event; a slot reused in the
        // meantime has harvested its owner under the lock first).
        if (b->done) cudaEventSynchronize(b->done);
        std::lock_guard<std::recursive_mutex> lock(g_mu);
        harvest(*b);
        std::vector<const void*> srcs;
        std::vector<void*> dsts;
        for (uint32_t i = 0; i < b->n; ++i) {
            if (b->status[i] == 1u) { ++g_verified; continue; }
            ++g_rejected;
            if (b->encrypted || b->items[i].src == nullptr) { ok = false; continue; }
            srcs.push_back(b->items[i].src);
            dsts.push_back(b->items[i].dst);
        }
        if (srcs.empty()) continue;
        // One strict retry from the trusted host copy under fresh tickets.
        g_retried += srcs.size();
        auto r = submit_layer_locked(b->layer, srcs.data(), dsts.data(), static_cast<uint32_t>(srcs.size()), b->count,
                                     b->codec.bits ? &b->codec : nullptr, false, nullptr, b->stream);
        if (!r) { ok = false; continue; }
        harvest(*r);
        for (uint32_t i = 0; i < r->n; ++i) {
            if (r->status[i] == 1u) ++g_verified; else { ++g_rejected; ok = false; }
        }
        std::lock_guard<std::mutex> ev(g_events_mu);
        g_s.last_event[b->layer] = r->done;
        g_s.last_batch[b->layer] = r;
    }
    return ok ? 0 : -1;
}

SI_EXPORT void secure_infer_recovery_set_job_id(uint64_t job_id)
{
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    g_s.job = job_id;
}

SI_EXPORT int secure_infer_recovery_wait_job_authentication(uint64_t job_id)
{
    std::vector<std::shared_ptr<LayerBatch>> batches;
    {
        std::lock_guard<std::recursive_mutex> lock(g_mu);
        for (auto it = g_s.pending.begin(); it != g_s.pending.end();) {
            auto& v = it->second;
            for (auto b = v.begin(); b != v.end();) {
                if ((*b)->job == job_id) { batches.push_back(*b); b = v.erase(b); } else { ++b; }
            }
            it = v.empty() ? g_s.pending.erase(it) : std::next(it);
        }
    }
    if (batches.empty()) return -1;
    bool valid = true;
    for (auto& b : batches)
        if (b->done) cudaEventSynchronize(b->done);
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    for (auto& b : batches) {
        harvest(*b);
        for (uint32_t i = 0; i < b->n; ++i) {
            if (b->status[i] == 1u) ++g_verified; else { ++g_rejected; valid = false; }
        }
    }
    return valid ? 1 : 0;
}

SI_EXPORT int secure_infer_d2h_batch_begin(size_t expected_groups)
{
    (void)expected_groups;
    std::lock_guard<std::mutex> dl(g_d2h_mu);
    t_d2h_batch = ++g_d2h_batch_id;
    return 0;
}

SI_EXPORT int secure_infer_d2h_group_begin(size_t expected_tasks)
{
    if (t_d2h_group_depth++ == 0) {
        t_d2h_group.clear();
        t_d2h_group.reserve(expected_tasks);
    }
    return 0;
}

SI_EXPORT int secure_infer_d2h_submit(void* dst_host, const void* src_device, size_t count, void* stream)
{
    if (dst_host == nullptr || src_device == nullptr || count == 0) return -1;
    t_d2h_group.push_back({dst_host, src_device, count, static_cast<cudaStream_t>(stream)});
    if (t_d2h_group_depth == 0) return d2h_flush_thread_group();
    return 0;
}

SI_EXPORT int secure_infer_d2h_group_end(void)
{
    if (t_d2h_group_depth == 0) return -1;
    if (--t_d2h_group_depth != 0) return 0;
    return d2h_flush_thread_group();
}

SI_EXPORT int secure_infer_d2h_batch_device_barrier(void) { return d2h_join(t_d2h_batch, true); }

SI_EXPORT int secure_infer_d2h_batch_end(void)
{
    const int rc = d2h_join(t_d2h_batch, false);
    t_d2h_batch = 0;
    return rc;
}

SI_EXPORT int secure_infer_d2h_writeback_layer(const void* const* src_blocks, void* const* dsts, uint32_t n,
                                               const secure_infer_codec* codec, void* stream)
{
    if (codec == nullptr) return -1;
    const uint64_t raw = 2ull * 128u * codec->heads * 128u;
    return d2h_submit_group(src_blocks, dsts, n, raw, codec, static_cast<cudaStream_t>(stream));
}

SI_EXPORT int secure_infer_d2h_wait(void) { return d2h_join(0, false); }

SI_EXPORT uint32_t secure_infer_set_layer_sm_limit(uint32_t sms) { return sib::set_layer_sm_limit(sms); }

SI_EXPORT int secure_infer_kernel_profile_enable(int on)
{
    sib::profile_enable(on != 0);
    return 0;
}

SI_EXPORT int secure_infer_kernel_profile_collect(double* total_us, uint64_t* launches, uint32_t kinds)
{
    return sib::profile_collect(total_us, launches, kinds);
}

SI_EXPORT const char* secure_infer_kernel_name(uint32_t kind) { return sib::kernel_kind_name(kind); }

SI_EXPORT int secure_infer_writeback_records(const void* const* srcs, void* const* host_dsts, uint32_t n,
                                             const secure_infer_codec* codec, void* records, uint64_t record_stride,
                                             uint64_t* tickets_out, void* stream)
{
    sib::CodecParams cp;
    uint64_t packet = 0;
    if (codec == nullptr || srcs == nullptr || records == nullptr || tickets_out == nullptr || n == 0 ||
        !codec_geometry(codec, &cp, &packet, true))
        return -1;
    const uint64_t count = cp.bits ? packet : 2ull * 128u * codec->heads * 128u;
    if (codec->heads == 0 || record_stride < record_bytes(count) || (record_stride & 15u) ||
        (cp.bits && cp.kind == SECURE_INFER_KIND_KV && (n & 1u)))
        return -1;
    for (uint32_t i = 0; i < n; ++i)
        if (srcs[i] == nullptr) return -1;
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (!g_s.ready) return -1;
    StageSlot& slot = g_s.wb[g_s.wb_next];
    g_s.wb_next = (g_s.wb_next + 1) % g_s.wb.size();
    if (slot.done) cudaEventSynchronize(slot.done);   // its pinned AAD copy and scratch are free
    if (!slot.done && !CUDA_OK(cudaEventCreateWithFlags(&slot.done, cudaEventDisableTiming))) return -1;
    if (!ensure_stage(slot, 16, sib::layer_ks_stride(count) * n, n, cp.bits ? packet * n : 0)) return -1;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (writeback_device_locked(srcs, host_dsts, n, cp, codec->layer, count, static_cast<uint8_t*>(records),
                                record_stride, slot, tickets_out, nullptr, nullptr, s) != 0)
        return -1;
    return CUDA_OK(cudaEventRecord(slot.done, s)) ? 0 : -1;
}

SI_EXPORT void secure_infer_invalidate_transfer_prefetches(void)
{
    ++g_generation;
    prep_drop_stale();
}

SI_EXPORT void secure_infer_retire_transfer_prefetches(void)
{
    ++g_generation;
    prep_drop_stale();
}

SI_EXPORT void secure_infer_get_transfer_prefetch_stats(uint64_t* ready, uint64_t* busy_fallback,
                                                        uint64_t* missing_fallback)
{
    if (ready) *ready = g_prep_ready.load();
    if (busy_fallback) *busy_fallback = g_prep_busy.load();
    if (missing_fallback) *missing_fallback = g_prep_missing.load();
}

SI_EXPORT void secure_infer_get_gcm_keystream_stats(uint64_t* scheduled, uint64_t* ready, uint64_t* hit,
                                                    uint64_t* miss, uint64_t* retired, uint64_t* stale,
                                                    uint64_t* failed)
{
    if (scheduled) *scheduled = g_ks_scheduled.load();
    if (ready) *ready = g_ks_scheduled.load();
    if (hit) *hit = g_ks_hit.load();
    if (miss) *miss = 0;
    if (retired) *retired = g_ks_hit.load();
    if (stale) *stale = 0;
    if (failed) *failed = 0;
}

SI_EXPORT void secure_infer_get_npu_keystream_stats(uint64_t* launched, uint64_t* completed, uint64_t* failed)
{
    if (launched) *launched = g_ks_launches.load();
    if (completed) *completed = g_ks_launches.load();
    if (failed) *failed = 0;
}

SI_EXPORT void secure_infer_get_npu_keystream_pool_stats(uint64_t* slots, uint64_t* in_use)
{
    std::lock_guard<std::recursive_mutex> lock(g_mu);
    if (slots) *slots = g_s.h2d.size();
    if (in_use) {
        uint64_t u = 0;
        for (auto& s : g_s.h2d) u += (s.owner && !s.owner->harvested) ? 1 : 0;
        *in_use = u;
    }
}

SI_EXPORT uint64_t secure_infer_count_ready_unconsumed_gcm_tickets(void) { return 0; }
SI_EXPORT int secure_infer_flush_completed_h2d_profile(void) { return 0; }
SI_EXPORT int secure_infer_drain_h2d_profile_after_job(void) { return 0; }

SI_EXPORT void secure_infer_get_auth_stats(uint64_t* verified, uint64_t* rejected, uint64_t* retried)
{
    if (verified) *verified = g_verified.load();
    if (rejected) *rejected = g_rejected.load();
    if (retried) *retried = g_retried.load();
}

SI_EXPORT void secure_infer_arm_tamper(uint32_t direction, uint64_t nth, uint32_t target)
{
    if (direction == SECURE_INFER_DIRECTION_H2D) {
        g_tamper_h2d_target = target;
        g_tamper_h2d_nth = nth;
    } else if (direction == SECURE_INFER_DIRECTION_D2H) {
        g_tamper_d2h_nth = nth;
    }
}
