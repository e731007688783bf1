// gcm_kernels.cuh -- launch descriptors shared by the CUDA kernels
// (gcm_kernels.cu) and the host runtime (host_runtime.cpp).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace sib {

struct GcmSchedule;  // gcm_device.cuh

// One authenticated record.  Segment work items are assigned in record order;
// seg_first is the record's first work item (exclusive prefix sum of nseg).
enum : uint32_t {
    kOpDecrypt = 1,   // in = C -> out = P (zeroed on failure), status
    kOpVerify = 2,    // in = C -> status only
    kOpEncrypt = 3,   // in = P -> out = C, tag_out = GHASH(C) ^ E_K(J0)
    kOpGhash = 4,     // generic GHASH (flags below), ghash_do semantics
    kOpXorOnly = 5,   // out = in ^ ks, status = 1, no authentication
};
enum : uint32_t {
    kGhashFinalize = 1u << 0,
    kGhashVerify = 1u << 1,
    kGhashXorOnSuccess = 1u << 2,
    kRecUnaligned = 1u << 8,   // some pointer is not 16-byte aligned
};

struct GcmRecord {
    const uint8_t* in;
    const uint8_t* ks;         // keystream for in[0..count), or null (AES inline)
    const uint8_t* aad;
    const uint8_t* tag_in;     // expected tag (verify paths)
    const uint8_t* tag_mask;   // explicit tag mask (kOpGhash + kGhashFinalize)
    uint8_t* out;
    uint8_t* tag_out;
    uint32_t* status;
    uint64_t count;
    uint32_t iv[4];            // big-endian packs of the IV bytes; iv[3] = first counter
    uint32_t aad_bytes;
    uint32_t op;
    uint32_t flags;
    uint32_t seg_first;
    uint32_t nseg;
    uint32_t reserved;
};

// KV codec geometry of a layer launch (one bit width per launch).
struct CodecParams {
    uint32_t bits;    // 8 or 4
    uint32_t kind;    // 0 = K (64-token groups per channel), 1 = V (64-dim groups)
    uint32_t heads;   // KV heads in one block; head_dim is 128, tokens 128
    uint32_t qb;      // quantised bytes
    uint32_t sb;      // bytes of one fp32 parameter array (scale or low)
};

constexpr int kInlineRecords = 4;

struct SegmentLaunch {
    const GcmSchedule* sched;
    const GcmRecord* recs;              // device array, or null -> inl
    GcmRecord inl[kInlineRecords];
    uint32_t nrec;
    uint32_t total_segs;
    uint4* partials;                    // [total_segs]
    uint32_t* counters;                 // [nrec], zero on entry, zero on exit
    uint32_t seg_blocks;                // segment length: 256..4096 (power of two); 0 = 4096
};

// AES-CTR keystream / CTR XOR jobs.
struct CtrJob {
    const uint8_t* in;   // null -> keystream only
    uint8_t* out;
    uint64_t bytes;
    uint32_t iv[4];
    uint64_t block_first;  // exclusive prefix sum of ceil(bytes/16)
};

constexpr int kInlineCtrJobs = 32;

struct CtrLaunch {
    const GcmSchedule* sched;
    const CtrJob* jobs;                 // device array, or null -> inl
    CtrJob inl[kInlineCtrJobs];
    uint32_t njobs;
    uint32_t unaligned;
    uint64_t total_blocks;
};

// KV codec encode (writeback quantisation) of n blocks of one layer/kind.
struct EncodeLaunch {
    const uint8_t* const* srcs;    // device array [n] of bf16 blocks (128 x heads x 128)
    uint8_t* packets;              // [n][width]
    uint32_t n;
    uint32_t width;
    uint32_t layer;
    CodecParams codec;
    uint32_t v_first;              // records r >= v_first are V blocks, the rest K
};

// A layer of uniform records laid out as C[aligned32(count)] || tag || 0^16 ||
// AAD64 at `records + i * stride`, IV = {iv0, ticket >> 32, ticket, 2}.  Passed
// by value in kernel parameters (16 bytes per record), so a launch needs no
// descriptor copy.  Keystream record i lives at ks + i * ks_stride,
// ks_stride = round16(count) + 16, with E_K(J0) in its last 16 bytes.
struct LayerRec {
    uint8_t* dst;
    uint64_t ticket;
};

struct LayerHeader {
    const GcmSchedule* sched;
    const uint8_t* records;
    uint64_t stride;
    uint64_t count;
    uint8_t* ks;
    uint64_t ks_stride;
    uint32_t* status;
    uint4* partials;        // [n * nseg]
    uint32_t* counters;     // [n], zero on entry and exit
    uint32_t iv0;
    uint32_t n;
    uint32_t nseg;          // segments per record
    uint32_t seg_steps;     // segment = 32 * seg_steps blocks (1..64)
    uint32_t unaligned;
    CodecParams codec;      // bits 0: raw payload; 8/4: codec packets dequantised into bf16 blocks
    uint32_t v_first;       // codec: records r >= v_first decode as V packets, the rest as K
    const uint8_t* aad;     // encrypt: AAD of record r at aad + 64 r (records are the output)
    const uint4* join_pow;  // H^(32 seg_steps 2^b) nibble tables, b = 1..5 (join_tables_for)
    // AES-128 round keys (LE words, as GcmSchedule::rk): read by the layer
    // kernels from the kernel parameters, i.e. the constant bank, so a round
    // key costs no shared-memory load and no register.
    uint32_t rk[44];
};

template <int kCap>
struct LayerLaunch {
    LayerHeader h;
    LayerRec rec[kCap];
};

constexpr int kLayerCapSmall = 128;
constexpr int kLayerCapLarge = 1024;

inline uint64_t layer_ks_stride(uint64_t count) { return ((count + 15) & ~uint64_t(15)) + 16; }
// Segment length (seg_steps) and count (nseg) per record for a launch of n records.
void layer_segments_for(uint64_t count, uint32_t n, uint32_t codec_bits, uint32_t* seg_steps, uint32_t* nseg);
// SMs a layer launch may occupy from now on (0: all of them); returns the
// previous limit.
uint32_t set_layer_sm_limit(uint32_t sms);

// Keystream (+ tag masks) and fused verify/XOR/scatter for up to
// kLayerCapLarge records; rec points at n LayerRec entries.  The encrypt
// launch is the writeback mirror: rec[i].dst is the plaintext (raw block or
// codec packet) of record i, written as C || tag || 0^16 || AAD into
// records + i * stride.
int launch_layer_keystream(const LayerHeader& h, const LayerRec* rec, cudaStream_t stream);
int launch_layer_verify(const LayerHeader& h, const LayerRec* rec, cudaStream_t stream);
int launch_layer_encrypt(const LayerHeader& h, const LayerRec* rec, cudaStream_t stream);
// Fused verify with the AES keystream computed in the kernel (h.ks unused):
// raw payloads (codec.bits 0), 16-byte aligned records and destinations.
int launch_layer_verify_inline(const LayerHeader& h, const LayerRec* rec, cudaStream_t stream);

// Kernel profile: while enabled, every launch below is bracketed by timing
// events on its stream; collect() sums device time and launches per kind.
enum KernelKind : uint32_t {
    kKernLayerCtr = 0, kKernLayerVerify, kKernLayerEncrypt, kKernEncode, kKernSegment, kKernCtr, kKernSchedule,
    kKernAuthGate, kKernLayerVerifyInline, kKernLayerCtrBitsliced, kKernKinds
};
void profile_enable(bool on);
int profile_collect(double* total_us, uint64_t* launches, uint32_t kinds);
const char* kernel_kind_name(uint32_t kind);

// Host-side launchers (gcm_kernels.cu).  Return a cudaError_t value.
// key may be null (GHASH-only requests); h null -> H = E_K(0^128) on device.
int launch_schedule(GcmSchedule* sched, const void* key, const void* h, bool need_tables, cudaStream_t stream);

// Segment join tables of the layer kernels for a session schedule: 64 segment
// lengths x 5 powers x 8 KiB (join_tables_bytes()).  LayerHeader::join_pow for
// a launch with seg_steps s is join_tables_for(tables, s).
constexpr size_t join_tables_bytes() { return 64u * 5u * 512u * 16u; }
inline const uint4* join_tables_for(const void* tables, uint32_t seg_steps)
{
    return static_cast<const uint4*>(tables) + (seg_steps - 1u) * 5u * 512u;
}
int launch_join_tables(const GcmSchedule* sched, void* out, cudaStream_t stream);
int launch_ctr(const CtrLaunch& args, cudaStream_t stream);
int launch_ctr_uniform(const CtrLaunch& args, uint64_t uniform_blocks, cudaStream_t stream);
int launch_auth_gate(uint8_t* data, const uint32_t* status, uint64_t bytes, cudaStream_t stream);
// Device half of the X25519/BLAKE2b session key agreement (32-byte publics,
// challenge and proof; 16-byte key; status 0 = done).
int launch_key_agreement(const void* host_public, const void* challenge, void* device_key, void* device_public,
                         void* proof, int32_t* status, cudaStream_t stream);
int launch_segments(const SegmentLaunch& args, bool inline_aes, cudaStream_t stream);
int launch_encode(const EncodeLaunch& args, cudaStream_t stream);
size_t schedule_bytes();
uint32_t segments_for(uint64_t count, uint32_t aad_bytes, uint32_t seg_blocks = 4096);
// Segment length for a segment-kernel launch covering `total_blocks` 16-byte
// blocks: the longest of 4096 .. 256 that still gives every SM two segments.
uint32_t segment_blocks_for(uint64_t total_blocks);


}  // namespace sib
