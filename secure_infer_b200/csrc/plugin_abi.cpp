// plugin_abi.cpp -- the GHASH_LIBRARY plugin ABI on CUDA streams.
//
// Exports the entry points the reference's data plane binds from its device
// crypto plugin (secure_infer/native/kernels/aicpu/launcher.asc:23-524,
// declared by secure_infer/native/secure_infer.h:396-457), with the same
// names, argument order, argument meaning and return convention:
//   * every pointer except `stream` is a device pointer;
//   * the work is enqueued on `stream` (a cudaStream_t; nullptr is CUDA's
//     legacy default stream, which is a valid stream here);
//   * the call returns 0 once the work is enqueued, -1 for null/zero
//     arguments or an unsupported size, and never blocks on the device;
//   * outputs are plaintext, or zeros when the tag does not verify; `status`
//     receives uint32 1 (authentic) or 0.
// Arguments are passed to the kernel by value (kernel parameter space), so
// nothing the caller passes has to outlive the call.
//
// Scratch: each (device, stream) pair owns one device scratch area (a key
// schedule of ~330 KB plus segment partials and counters), allocated with
// cudaMalloc on the first call that uses that stream and kept until exit.  The
// first call on a stream therefore allocates and should happen before any
// stream capture.  The schedule is rebuilt on the device only when the key or
// H bytes change.
#include "gcm_kernels.cuh"
#include "../../include/secure_infer_gcm_plugin.h"

#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

namespace sib {
namespace {

constexpr uint32_t kScratchSegments = 1u << 16;   // 4 GiB of payload per call
constexpr uint32_t kScratchRecords = 64;

struct StreamScratch {
    int device = -1;
    cudaStream_t stream = nullptr;
    GcmSchedule* sched = nullptr;
    uint4* partials = nullptr;
    uint32_t* counters = nullptr;
};

std::mutex g_scratch_mu;
std::vector<std::unique_ptr<StreamScratch>> g_scratch;

StreamScratch* scratch_for(cudaStream_t stream)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    for (auto& s : g_scratch)
        if (s->device == dev && s->stream == stream) return s.get();
    auto s = std::make_unique<StreamScratch>();
    s->device = dev;
    s->stream = stream;
    if (cudaMalloc(&s->sched, schedule_bytes()) != cudaSuccess ||
        cudaMalloc(&s->partials, sizeof(uint4) * kScratchSegments) != cudaSuccess ||
        cudaMalloc(&s->counters, sizeof(uint32_t) * kScratchRecords) != cudaSuccess ||
        cudaMemset(s->sched, 0, schedule_bytes()) != cudaSuccess ||
        cudaMemset(s->counters, 0, sizeof(uint32_t) * kScratchRecords) != cudaSuccess) {
        cudaFree(s->sched);
        cudaFree(s->partials);
        cudaFree(s->counters);
        return nullptr;
    }
    g_scratch.push_back(std::move(s));
    return g_scratch.back().get();
}

bool misaligned(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; }

GcmRecord make_record(uint32_t op, const void* in, const void* ks, const void* aad, uint64_t aad_bytes,
                      const void* tag_in, void* out, void* tag_out, void* status, uint64_t bytes,
                      uint32_t iv0, uint32_t iv1, uint32_t iv2, uint32_t iv3)
{
    GcmRecord r{};
    r.op = op;
    r.in = static_cast<const uint8_t*>(in);
    r.ks = static_cast<const uint8_t*>(ks);
    r.aad = static_cast<const uint8_t*>(aad_bytes ? aad : nullptr);
    r.aad_bytes = static_cast<uint32_t>(aad_bytes);
    r.tag_in = static_cast<const uint8_t*>(tag_in);
    r.out = static_cast<uint8_t*>(out);
    r.tag_out = static_cast<uint8_t*>(tag_out);
    r.status = static_cast<uint32_t*>(status);
    r.count = bytes;
    r.iv[0] = iv0; r.iv[1] = iv1; r.iv[2] = iv2; r.iv[3] = iv3;
    if (misaligned(in) || misaligned(ks) || misaligned(out)) r.flags |= kRecUnaligned;
    return r;
}

// Enqueue schedule + one segmented launch over up to kInlineRecords records.
int run_records(cudaStream_t stream, const void* key, const void* h, GcmRecord* recs, uint32_t n)
{
    StreamScratch* s = scratch_for(stream);
    if (s == nullptr || n == 0 || n > static_cast<uint32_t>(kInlineRecords)) return -1;
    SegmentLaunch L{};
    uint32_t total = 0;
    bool inline_aes = false;
    // A call carries one to four records: shorter segments keep the SMs busy
    // when the payload is small (one 256 KiB record -> 16 segments).
    uint64_t blocks = 0;
    for (uint32_t i = 0; i < n; ++i)
        blocks += (recs[i].aad_bytes + 15u) / 16u + (recs[i].count + 15u) / 16u + 1u;
    L.seg_blocks = segment_blocks_for(blocks);
    for (uint32_t i = 0; i < n; ++i) {
        if (recs[i].aad_bytes > (1u << 20)) return -1;
        const bool needs_ks = recs[i].op == kOpDecrypt || recs[i].op == kOpEncrypt;
        inline_aes = inline_aes || (needs_ks && recs[i].ks == nullptr);
        recs[i].seg_first = total;
        recs[i].nseg = segments_for(recs[i].count, recs[i].aad_bytes, L.seg_blocks);
        total += recs[i].nseg;
        L.inl[i] = recs[i];
    }
    if (total > kScratchSegments) return -1;
    if (launch_schedule(s->sched, key, h, true, stream) != cudaSuccess) return -1;
    L.sched = s->sched;
    L.recs = nullptr;
    L.nrec = n;
    L.total_segs = total;
    L.partials = s->partials;
    L.counters = s->counters;
    return launch_segments(L, inline_aes, stream) == cudaSuccess ? 0 : -1;
}

int run_ctr(cudaStream_t stream, const void* key, const CtrJob* jobs, uint32_t n)
{
    StreamScratch* s = scratch_for(stream);
    if (s == nullptr || n == 0 || n > static_cast<uint32_t>(kInlineCtrJobs)) return -1;
    if (launch_schedule(s->sched, key, nullptr, false, stream) != cudaSuccess) return -1;
    CtrLaunch L{};
    L.sched = s->sched;
    L.jobs = nullptr;
    L.njobs = n;
    uint64_t total = 0;
    for (uint32_t i = 0; i < n; ++i) {
        L.inl[i] = jobs[i];
        L.inl[i].block_first = total;
        total += (jobs[i].bytes + 15) / 16;
        if (misaligned(jobs[i].in) || misaligned(jobs[i].out)) L.unaligned = 1;
    }
    L.total_blocks = total;
    return launch_ctr(L, stream) == cudaSuccess ? 0 : -1;
}

}  // namespace
}  // namespace sib

using namespace sib;

#define SI_EXPORT extern "C" __attribute__((visibility("default")))

SI_EXPORT int secure_infer_aicpu_ghash_do(void* stream, void* input, void* hash_subkey, void* output, void* aad,
                                          void* tag_mask, void* expected_tag, void* keystream,
                                          void* plaintext_output, void* status_output, uint64_t input_bytes,
                                          uint64_t aad_bytes, uint32_t flags)
{
    if (input == nullptr || hash_subkey == nullptr || output == nullptr || input_bytes == 0) return -1;
    if ((aad_bytes != 0 && aad == nullptr) || ((flags & kGhashFinalize) && tag_mask == nullptr) ||
        ((flags & kGhashVerify) && expected_tag == nullptr) ||
        ((flags & kGhashXorOnSuccess) && (keystream == nullptr || plaintext_output == nullptr)))
        return -1;
    GcmRecord r = make_record(kOpGhash, input, (flags & kGhashXorOnSuccess) ? keystream : nullptr, aad, aad_bytes,
                              expected_tag, (flags & kGhashXorOnSuccess) ? plaintext_output : nullptr, output,
                              status_output, input_bytes, 0, 0, 0, 0);
    r.flags |= flags & (kGhashFinalize | kGhashVerify | kGhashXorOnSuccess);
    r.tag_mask = static_cast<const uint8_t*>(tag_mask);
    return run_records(static_cast<cudaStream_t>(stream), nullptr, hash_subkey, &r, 1);
}

SI_EXPORT int secure_infer_aicpu_auth_gate_do(void* stream, void* data, void* status, uint64_t bytes)
{
    if (data == nullptr || status == nullptr || bytes == 0) return -1;
    return launch_auth_gate(static_cast<uint8_t*>(data), static_cast<const uint32_t*>(status), bytes,
                            static_cast<cudaStream_t>(stream)) == cudaSuccess ? 0 : -1;
}

SI_EXPORT int secure_infer_aicpu_key_agreement_do(void* stream, void* host_public, void* challenge, void* device_key,
                                                  void* device_public, void* proof, void* status)
{
    if (host_public == nullptr || challenge == nullptr || device_key == nullptr || device_public == nullptr ||
        proof == nullptr || status == nullptr)
        return -1;
    return launch_key_agreement(host_public, challenge, device_key, device_public, proof,
                                static_cast<int32_t*>(status), static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? 0
               : -1;
}

SI_EXPORT int secure_infer_aicpu_aes_ctr_do(void* stream, void* input, void* key, void* output, uint64_t bytes,
                                            uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2,
                                            uint32_t iv_word3)
{
    if (input == nullptr || key == nullptr || output == nullptr || bytes == 0) return -1;
    CtrJob j{};
    j.in = static_cast<const uint8_t*>(input);
    j.out = static_cast<uint8_t*>(output);
    j.bytes = bytes;
    j.iv[0] = iv_word0; j.iv[1] = iv_word1; j.iv[2] = iv_word2; j.iv[3] = iv_word3;
    return run_ctr(static_cast<cudaStream_t>(stream), key, &j, 1);
}

SI_EXPORT int secure_infer_aicpu_keystream_do(void* stream, void* key, void* output, uint64_t bytes,
                                              uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2,
                                              uint32_t iv_word3)
{
    if (key == nullptr || output == nullptr || bytes == 0) return -1;
    CtrJob j{};
    j.out = static_cast<uint8_t*>(output);
    j.bytes = bytes;
    j.iv[0] = iv_word0; j.iv[1] = iv_word1; j.iv[2] = iv_word2; j.iv[3] = iv_word3;
    return run_ctr(static_cast<cudaStream_t>(stream), key, &j, 1);
}

SI_EXPORT int secure_infer_aicpu_keystream_batch_do(void* stream, void* key, void* const* outputs,
                                                    const uint32_t* iv_words, uint64_t bytes, uint32_t count)
{
    if (key == nullptr || outputs == nullptr || iv_words == nullptr || bytes == 0 || count == 0 ||
        count > SECURE_INFER_KEYSTREAM_BATCH_MAX)
        return -1;
    CtrJob jobs[kInlineCtrJobs] = {};
    for (uint32_t i = 0; i < count; ++i) {
        if (outputs[i] == nullptr) return -1;
        jobs[i].out = static_cast<uint8_t*>(outputs[i]);
        jobs[i].bytes = bytes;
        for (int w = 0; w < 4; ++w) jobs[i].iv[w] = iv_words[4 * i + w];
    }
    return run_ctr(static_cast<cudaStream_t>(stream), key, jobs, count);
}

SI_EXPORT int secure_infer_aicpu_gcm_decrypt_verify_aad_do(void* stream, void* ciphertext, void* key,
                                                           void* hash_subkey, void* expected_tag,
                                                           void* plaintext_output, void* status_output,
                                                           uint64_t bytes, uint32_t iv_word0, uint32_t iv_word1,
                                                           uint32_t iv_word2, uint32_t iv_word3, void* aad,
                                                           uint64_t aad_bytes)
{
    if (ciphertext == nullptr || key == nullptr || hash_subkey == nullptr || expected_tag == nullptr ||
        plaintext_output == nullptr || status_output == nullptr || bytes == 0 || (aad_bytes != 0 && aad == nullptr))
        return -1;
    GcmRecord r = make_record(kOpDecrypt, ciphertext, nullptr, aad, aad_bytes, expected_tag, plaintext_output,
                              nullptr, status_output, bytes, iv_word0, iv_word1, iv_word2, iv_word3);
    return run_records(static_cast<cudaStream_t>(stream), key, hash_subkey, &r, 1);
}

SI_EXPORT int secure_infer_aicpu_gcm_decrypt_verify_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                                       void* expected_tag, void* plaintext_output,
                                                       void* status_output, uint64_t bytes, uint32_t iv_word0,
                                                       uint32_t iv_word1, uint32_t iv_word2, uint32_t iv_word3)
{
    return secure_infer_aicpu_gcm_decrypt_verify_aad_do(stream, ciphertext, key, hash_subkey, expected_tag,
                                                        plaintext_output, status_output, bytes, iv_word0, iv_word1,
                                                        iv_word2, iv_word3, nullptr, 0);
}

SI_EXPORT int secure_infer_aicpu_gcm_encrypt_tag_do(void* stream, void* plaintext, void* key, void* hash_subkey,
                                                    void* ciphertext_output, void* tag_output, uint64_t bytes,
                                                    uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2,
                                                    uint32_t iv_word3, void* aad, uint64_t aad_bytes)
{
    if (plaintext == nullptr || key == nullptr || hash_subkey == nullptr || ciphertext_output == nullptr ||
        tag_output == nullptr || bytes == 0 || (aad_bytes != 0 && aad == nullptr))
        return -1;
    GcmRecord r = make_record(kOpEncrypt, plaintext, nullptr, aad, aad_bytes, nullptr, ciphertext_output, tag_output,
                              nullptr, bytes, iv_word0, iv_word1, iv_word2, iv_word3);
    return run_records(static_cast<cudaStream_t>(stream), key, hash_subkey, &r, 1);
}

SI_EXPORT int secure_infer_aicpu_gcm_verify_xor_aad_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                                       void* expected_tag, void* keystream, void* plaintext_output,
                                                       void* status_output, uint64_t bytes, uint32_t iv_word0,
                                                       uint32_t iv_word1, uint32_t iv_word2, uint32_t iv_word3,
                                                       void* aad, uint64_t aad_bytes)
{
    if (ciphertext == nullptr || key == nullptr || hash_subkey == nullptr || expected_tag == nullptr ||
        keystream == nullptr || plaintext_output == nullptr || status_output == nullptr || bytes == 0 ||
        (aad_bytes != 0 && aad == nullptr))
        return -1;
    GcmRecord r = make_record(kOpDecrypt, ciphertext, keystream, aad, aad_bytes, expected_tag, plaintext_output,
                              nullptr, status_output, bytes, iv_word0, iv_word1, iv_word2, iv_word3);
    return run_records(static_cast<cudaStream_t>(stream), key, hash_subkey, &r, 1);
}

SI_EXPORT int secure_infer_aicpu_gcm_verify_xor_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                                   void* expected_tag, void* keystream, void* plaintext_output,
                                                   void* status_output, uint64_t bytes, uint32_t iv_word0,
                                                   uint32_t iv_word1, uint32_t iv_word2, uint32_t iv_word3)
{
    return secure_infer_aicpu_gcm_verify_xor_aad_do(stream, ciphertext, key, hash_subkey, expected_tag, keystream,
                                                    plaintext_output, status_output, bytes, iv_word0, iv_word1,
                                                    iv_word2, iv_word3, nullptr, 0);
}

SI_EXPORT int secure_infer_aicpu_gcm_verify_only_aad_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                                        void* expected_tag, void* status_output, uint64_t bytes,
                                                        uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2,
                                                        uint32_t iv_word3, void* aad, uint64_t aad_bytes)
{
    if (ciphertext == nullptr || key == nullptr || hash_subkey == nullptr || expected_tag == nullptr ||
        status_output == nullptr || bytes == 0 || (aad_bytes != 0 && aad == nullptr))
        return -1;
    GcmRecord r = make_record(kOpVerify, ciphertext, nullptr, aad, aad_bytes, expected_tag, nullptr, nullptr,
                              status_output, bytes, iv_word0, iv_word1, iv_word2, iv_word3);
    return run_records(static_cast<cudaStream_t>(stream), key, hash_subkey, &r, 1);
}

SI_EXPORT int secure_infer_aicpu_gcm_verify_only_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                                    void* expected_tag, void* status_output, uint64_t bytes,
                                                    uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2,
                                                    uint32_t iv_word3)
{
    return secure_infer_aicpu_gcm_verify_only_aad_do(stream, ciphertext, key, hash_subkey, expected_tag,
                                                     status_output, bytes, iv_word0, iv_word1, iv_word2, iv_word3,
                                                     nullptr, 0);
}

SI_EXPORT int secure_infer_aicpu_gcm_verify_xor_batch_do(void* stream, void* key, void* hash_subkey,
                                                         void* const* ciphertexts, void* const* expected_tags,
                                                         void* const* keystreams, void* const* plaintext_outputs,
                                                         void* const* status_outputs, void* const* aads,
                                                         uint64_t bytes, uint64_t aad_bytes, const uint32_t* iv_words,
                                                         uint32_t count)
{
    if (key == nullptr || hash_subkey == nullptr || ciphertexts == nullptr || expected_tags == nullptr ||
        keystreams == nullptr || plaintext_outputs == nullptr || status_outputs == nullptr || iv_words == nullptr ||
        bytes == 0 || (aad_bytes != 0 && aads == nullptr) || count == 0 || count > SECURE_INFER_VERIFY_XOR_BATCH_MAX)
        return -1;
    GcmRecord recs[kInlineRecords];
    for (uint32_t i = 0; i < count; ++i) {
        if (ciphertexts[i] == nullptr || expected_tags[i] == nullptr || keystreams[i] == nullptr ||
            plaintext_outputs[i] == nullptr || status_outputs[i] == nullptr ||
            (aad_bytes != 0 && aads[i] == nullptr))
            return -1;
        recs[i] = make_record(kOpDecrypt, ciphertexts[i], keystreams[i], aad_bytes ? aads[i] : nullptr, aad_bytes,
                              expected_tags[i], plaintext_outputs[i], nullptr, status_outputs[i], bytes,
                              iv_words[4 * i], iv_words[4 * i + 1], iv_words[4 * i + 2], iv_words[4 * i + 3]);
    }
    return run_records(static_cast<cudaStream_t>(stream), key, hash_subkey, recs, count);
}

SI_EXPORT int secure_infer_aicpu_gcm_xor_only_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                                 void* expected_tag, void* keystream, void* plaintext_output,
                                                 void* status_output, uint64_t bytes, uint32_t iv_word0,
                                                 uint32_t iv_word1, uint32_t iv_word2, uint32_t iv_word3)
{
    if (ciphertext == nullptr || key == nullptr || hash_subkey == nullptr || expected_tag == nullptr ||
        keystream == nullptr || plaintext_output == nullptr || status_output == nullptr || bytes == 0)
        return -1;
    GcmRecord r = make_record(kOpXorOnly, ciphertext, keystream, nullptr, 0, expected_tag, plaintext_output, nullptr,
                              status_output, bytes, iv_word0, iv_word1, iv_word2, iv_word3);
    return run_records(static_cast<cudaStream_t>(stream), key, hash_subkey, &r, 1);
}
