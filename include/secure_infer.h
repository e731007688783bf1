/*
 * secure_infer.h -- host ABI of libsecure_infer.so, CUDA (sm_100a) edition.
 *
 * The reference library is LD_PRELOADed and reached from Python through
 * ctypes.CDLL(None) (secure_infer/kv_offload/npu_predict.py:158-254,
 * native_layerwise.py:90-93, transport_codec.py:50,150).  Every name the
 * reference exports for the authenticated KV transfer path is kept here with
 * its signature and return convention; the vendor-memcpy interposition of the
 * reference (aclrtMemcpyAsync, secure_infer.cpp:7729) is replaced by explicit
 * submission calls (secure_infer_h2d_submit / secure_infer_d2h_submit) that a
 * connector makes instead of the per-block vendor copy, plus per-layer calls
 * that move a whole layer in one staged copy and one fused kernel.
 *
 * Streams are cudaStream_t passed as void*.  Host pointers are plain host
 * memory (pinned for the pool); device pointers are CUDA device memory on the
 * session's device.  Functions returning int use 0 = success, -1 = failure
 * unless stated otherwise.
 */
#ifndef SECURE_INFER_H
#define SECURE_INFER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SECURE_INFER_GCM_AAD_BYTES 64u        /* secure_infer.h:59 */
#define SECURE_INFER_DIRECTION_H2D 1u         /* secure_infer.h:61 */
#define SECURE_INFER_DIRECTION_D2H 2u         /* secure_infer.h:62 */

/* ---------------------------------------------------------------- session */

/* Install the session key (16 bytes, AES-128) and the 4-byte IV salt on
 * `device`, derive H = E_K(0^128) and the key schedule on the device.  Stands
 * in for the device key agreement (secure_infer.cpp:449-521), whose outputs
 * are exactly this key and salt.  This is the recommended session path.
 * Clears the replay set.  Tickets come from one counter per process that no
 * init resets (as the reference's, secure_infer.cpp:126, :264), so a second
 * session with the same key and salt never repeats a GCM nonce. */
int secure_infer_session_init(int device, const uint8_t* key16, const uint8_t* iv_salt4);

/* Experimental session setup by key agreement (secure_infer.cpp:449-521,
 * secure_infer_experimental_device_session): the host draws an X25519 secret
 * and a 32-byte challenge (OpenSSL RAND_bytes), the device kernel
 * (secure_infer_aicpu_key_agreement_do) returns its public value and a proof,
 * the host derives key = BLAKE2b-16(key = shared, "SecureInfer X25519 BLAKE2b
 * test v1" || host public || device public || challenge), checks the proof
 * BLAKE2b-32(key = key, challenge) in constant time and derives the salt
 * BLAKE2b-4(key = shared, "SecureInfer IV salt v1").  The device key schedule
 * is built from the device's own copy of the key.  Returns 0, or -1 with no
 * session when any step or the proof check fails.
 *
 * WEAK DEVICE ENTROPY: the reference's AICPU reads its X25519 secret from
 * /dev/urandom; a GPU has no entropy source, so the device secret here is a
 * BLAKE2b hash of %globaltimer / clock64 samples and an atomic counter.  Those
 * inputs are partly predictable and hold little entropy, and a guessed device
 * secret reveals the session key.  Use secure_infer_session_init with a key
 * from a real key exchange for anything but experiments. */
int secure_infer_session_init_key_agreement(int device);

/* Tear down the session (waits for in-flight work, frees staging). */
int secure_infer_session_shutdown(void);

/* ------------------------------------------------------- host KV ranges */

/* secure_infer.cpp:1093. Registers a host range without KV metadata. */
void secure_infer_register_host_range(const void* base, size_t bytes);

/* secure_infer.cpp:1066-1091. Registers a host KV tensor: records inside it
 * carry (layer, kind, block = offset / block_bytes) in their AAD. */
void secure_infer_register_host_range_ex(const void* base, size_t bytes, uint32_t layer_id, uint32_t tensor_kind,
                                         size_t block_bytes);

/* 1 when [ptr, ptr + bytes) lies inside one registered host range, else 0.
 * No separate reference export: it is the reference's internal check
 * host_prediction_in_same_range (secure_infer.cpp:7733-7737), which decides
 * whether an interposed copy takes the authenticated path; the opt-in
 * cudaMemcpyAsync interposer (libsecure_infer_interpose.so) calls it. */
int secure_infer_is_registered_host_range(const void* ptr, size_t bytes);

/* ------------------------------------------------------ record helpers */

/* Host worker pool of this process.  No counterpart in the reference, whose
 * CPU worker counts come from PIPE_D2H_CPU_WORKERS and friends
 * (secure_infer.cpp:2568-2577).  Ranks that share a host (LOCAL_WORLD_SIZE >
 * 1) split the CPU affinity set into equal disjoint slices (slice LOCAL_RANK)
 * and pin their OpenSSL workers to it; a lone rank uses every allowed CPU.
 * Writes the worker count to *threads (the calling thread encrypts as well),
 * up to max_cpus CPU ids of the slice to cpus, and 1 to *pinned when the
 * workers are pinned.  Returns the slice's CPU count, or -1 when threads is
 * null.  SECURE_INFER_CRYPTO_THREADS overrides the worker count and
 * SECURE_INFER_PIN_THREADS=0/1 the pinning. */
int secure_infer_host_pool_info(uint32_t* threads, int32_t* cpus, uint32_t max_cpus, uint32_t* pinned);

/* Next transfer ticket (secure_infer.cpp:262-272); never 0.  Tickets handed
 * out here or by secure_infer_h2d_encrypt_records are redeemable once by a
 * pre-encrypted reload; a replayed or never-issued ticket is rejected. */
uint64_t secure_infer_new_transfer_ticket(void);

/* IV = base[0..3] || BE64(session_nonce + ticket) || BE32(block_offset + 2)
 * (secure_infer.cpp:274-300, GCM mode: session nonce 0).  -1 on ticket 0. */
int secure_infer_derive_transfer_iv(const uint8_t* base_iv16, uint64_t ticket, uint64_t block_offset,
                                    uint8_t* out_iv16);

/* 64-byte AAD "SFAD" v1 (secure_infer.cpp:730-775) for `bytes` at host_ptr,
 * using the registered range that contains it.  -1 on bad arguments. */
int secure_infer_build_gcm_aad(const void* host_ptr, size_t bytes, uint8_t direction, uint64_t ticket,
                               uint64_t transfer_offset, uint8_t* out64);

/* Bytes of one record: C padded to 32 || tag16 || zero16 || AAD64
 * (secure_infer.cpp:6379-6388). */
uint64_t secure_infer_record_bytes(uint64_t count);

/* Host AES-128-GCM encrypt of n slices into records (OpenSSL EVP, worker
 * threads), each with a fresh ticket; tickets_out[i] receives the ticket.
 * records: n * record_stride bytes of host memory.  (secure_infer.cpp:6508-6537) */
int secure_infer_h2d_encrypt_records(const void* const* srcs, uint64_t count, uint32_t n, void* records,
                                     uint64_t record_stride, uint64_t* tickets_out);

/* --------------------------------------------------- KV codec geometry */

typedef struct {
    uint32_t bits;    /* 0 = KV_CODEC none (raw bf16 bytes), 8 = int8, 4 = int4 */
    uint32_t kind;    /* 0 = K, 1 = V (grouping axis); reloads also take
                         SECURE_INFER_KIND_KV: n even, records [0, n/2) are K
                         packets and [n/2, n) V packets of the same layer */
    uint32_t heads;   /* KV heads per 128-token block; head_dim is 128 */
    uint32_t layer;   /* written into the packet header on encode */
} secure_infer_codec;

#define SECURE_INFER_KIND_KV 2u

/* Packet row bytes for (heads, bits): q || scale || low || int32[4], padded
 * to 16 (transport_codec.py:35-41).  0 for bits not in {8, 4}. */
uint64_t secure_infer_codec_packet_bytes(uint32_t heads, uint32_t bits);

/* -------------------------------------------- reload (H2D) of one layer */

/* Device part of a layer reload over records already in device memory.
 * records: n records at `records + i * record_stride`; tickets[i] gives the
 * IV; dsts[i] is the destination (raw bytes, or a bf16 paged-cache block when
 * codec->bits != 0, where the payload is a codec packet).  The AES-CTR
 * keystream is generated on `producer_stream` (null: the session's producer
 * stream) into `keystream` (device, n * (round16(count) + 16) bytes: record i
 * at i * (round16(count) + 16), its last 16 bytes holding the tag mask
 * E_K(J0); null: AES is computed inside the fused kernel); on a separate
 * producer stream the keystream launch waits for the work the caller's stream
 * had queued (so one keystream buffer may serve consecutive calls), and the
 * caller's stream waits for the keystream.  Then one fused kernel verifies
 * every tag, XORs, dequantises and scatters, zeroing the destination of any
 * record that fails.  status[i] (device) receives 1/0.  Host arrays are
 * captured at call time. */
int secure_infer_reload_records(uint32_t layer, const void* records, uint64_t record_stride, uint64_t count,
                                uint32_t n, const uint64_t* tickets, void* const* dsts, void* keystream,
                                uint32_t* status, const secure_infer_codec* codec, void* stream,
                                void* producer_stream);

/* The two halves of secure_infer_reload_records, on one stream:
 * keystream for n tickets into `keystream` (record i at i * (round16(count) + 16),
 * tag mask E_K(J0) in its last 16 bytes),
 * and the fused verify/XOR/(dequant)/scatter with that keystream ready (null
 * keystream: AES computed inside the fused kernel; codec records need a
 * keystream). */
int secure_infer_keystream_records(const uint64_t* tickets, uint32_t n, uint64_t count, void* keystream,
                                   void* stream);
int secure_infer_verify_records(uint32_t layer, const void* records, uint64_t record_stride, uint64_t count,
                                uint32_t n, const uint64_t* tickets, void* const* dsts, const void* keystream,
                                uint32_t* status, const secure_infer_codec* codec, void* stream);

/* Full reload of one layer/kind: host encrypt (or pre-encrypted records when
 * `records_are_encrypted` = 1 and srcs[0] points at n records with
 * record_stride = secure_infer_record_bytes(count) and tickets given), staged
 * H2D copy, keystream + fused verify/dequant/scatter, status D2H, and a
 * pending authentication entry for `layer`. */
int secure_infer_h2d_reload_layer(uint32_t layer, const void* const* srcs, void* const* dsts, uint32_t n,
                                  uint64_t count, const secure_infer_codec* codec, int records_are_encrypted,
                                  const uint64_t* tickets, void* stream);

/* The connector's per-layer fetch loop (reuse/connector.py:222-331, as
 * `RuntimeWorker.fetch_serialized`) run by a library thread, so no reload of a
 * request waits for the caller's interpreter.  Layers first_layer ..
 * first_layer + nlayers - 1; layer i reloads the n records srcs[i*n ..
 * (i+1)*n) into dsts[i*n .. (i+1)*n) (K records first, as
 * secure_infer_h2d_reload_layer) with counts[i] bytes each and codecs[i]
 * (NULL: all raw; bits 0: raw layer), on `stream`, announcing layer i + 1
 * before reloading layer i when `lookahead` is set.  Returns at once (0, or
 * -1 on bad arguments); the arrays are copied.  For a layer of the request,
 * secure_infer_recovery_wait_layer_authentication and
 * secure_infer_layer_ready_wait first wait until the thread has submitted it
 * (-1 if that submission failed).  One request at a time: a new one, a
 * session init or shutdown first joins the previous.  No separate reference
 * export: the reference runs this loop in Python. */
int secure_infer_h2d_reload_layers_async(uint32_t first_layer, uint32_t nlayers, const void* const* srcs,
                                         void* const* dsts, uint32_t n, const uint64_t* counts,
                                         const secure_infer_codec* codecs, int lookahead, void* stream);
/* Joins the request's thread: 0, or -1 if a reload could not be submitted. */
int secure_infer_h2d_reload_layers_join(void);

/* Record the completion event of the last reload of `layer` on `stream`
 * (device-side release of attention; no host wait).  -1 if none. */
int secure_infer_layer_ready_wait(uint32_t layer, void* stream);

/* ------------------------------------- reference bracket + submission */

/* secure_infer.cpp:5883-5903: submissions between begin/end of the outermost
 * group are batched and flushed at end as per-layer reloads. */
int secure_infer_h2d_layer_group_begin(size_t expected_tasks);
int secure_infer_h2d_layer_group_end(void);

/* Replaces one interposed H2D vendor copy of a registered host range
 * (secure_infer.cpp:7729-7855): authenticated copy of `count` bytes from
 * host `src` to device `dst`.  Inside a group it is queued; outside it is
 * flushed immediately. */
int secure_infer_h2d_submit(void* dst, size_t dst_capacity, const void* src, size_t count, void* stream);

/* --------------------------------------------------- authentication */

/* secure_infer.cpp:7303-7333: waits for every record of `layer`; a record
 * that failed is retried once from the trusted host copy with a fresh ticket;
 * 0 = all authentic, -1 = failure.  0 when nothing is pending. */
int secure_infer_recovery_wait_layer_authentication(uint32_t layer);

/* secure_infer.cpp:5311: job id attached to subsequent reloads. */
void secure_infer_recovery_set_job_id(uint64_t job_id);

/* secure_infer.cpp:7338: 1 = all records of the job authentic, 0 = some
 * failed, -1 = no records for the job. */
int secure_infer_recovery_wait_job_authentication(uint64_t job_id);

/* ---------------------------------------------- writeback (D2H) path */

/* secure_infer.cpp:2707-2970. Batch / group brackets; submissions inside a
 * group are encrypted and tagged on the device, copied to the host, verified
 * by host worker threads and decrypted into their destinations. */
int secure_infer_d2h_batch_begin(size_t expected_groups);
int secure_infer_d2h_group_begin(size_t expected_tasks);
int secure_infer_d2h_submit(void* dst_host, const void* src_device, size_t count, void* stream);
int secure_infer_d2h_group_end(void);
int secure_infer_d2h_batch_device_barrier(void);   /* device copies landed */
int secure_infer_d2h_batch_end(void);              /* host verification done */

/* Writeback of one layer/kind in one call: gather n bf16 blocks (src_blocks,
 * device), quantise with `codec` (bits 0 = raw), encrypt + tag on device,
 * copy to the host, verify on the host and store the packet (or raw bytes) to
 * dsts[i] (host, inside a registered range).  Returns after the device work is
 * enqueued; completion is joined by secure_infer_d2h_wait(). */
int secure_infer_d2h_writeback_layer(const void* const* src_blocks, void* const* dsts, uint32_t n,
                                     const secure_infer_codec* codec, void* stream);
int secure_infer_d2h_wait(void);

/* Device half of a writeback, the mirror of secure_infer_reload_records (no
 * single reference function: it is the device part of the D2H path,
 * ghash.aicpu:656-699 encrypt_tag after transport_codec.py:22-42 encode).
 * srcs[i]: device bf16 block (128 tokens x heads x 128); for codec bits 8/4
 * the blocks are quantised into packets first (kind 0 = K, 1 = V,
 * SECURE_INFER_KIND_KV = first n/2 K, rest V).  Each record gets a fresh
 * ticket (tickets_out[i], host) and its AAD names host_dsts[i] (the host-pool
 * slot it is meant for; may be null) with direction D2H.  Records
 * C || tag || 0^16 || AAD (count = packet bytes, or 2*128*heads*128 raw) go to
 * `records` (device, record_stride >= secure_infer_record_bytes(count)),
 * ordered on `stream`; they reload through secure_infer_reload_records. */
int secure_infer_writeback_records(const void* const* srcs, void* const* host_dsts, uint32_t n,
                                   const secure_infer_codec* codec, void* records, uint64_t record_stride,
                                   uint64_t* tickets_out, void* stream);

/* ------------------------------------------------------ SM share */

/* No reference counterpart.  The number of SMs each layer launch (keystream,
 * fused verify / inline-keystream verify, writeback encrypt) may occupy from
 * now on, process-wide; 0 (the default) means every SM.  The layer kernels
 * hold most of an SM's shared memory, so launches from different streams
 * otherwise queue for the same SMs.  A caller that alternates consecutive
 * layers between k streams sets it to about SMs / k so those launches run
 * side by side: measured on a B200 with two streams and half the SMs each,
 * 46.3 us per Llama-3-8B layer (8 KV heads, 6144 tokens) against 51.8 on one
 * stream with all SMs, and 10.9 against 15.4 us at one KV head.  Set it
 * between calls; a launch reads it once.  Returns the previous limit. */
uint32_t secure_infer_set_layer_sm_limit(uint32_t sms);

/* ------------------------------------------------------ kernel profile */

/* No reference counterpart (the reference's h2d profile hooks below print
 * transfer timings): while enabled, every kernel launch of this library is
 * bracketed by CUDA timing events on its stream.  collect() waits for the
 * recorded launches, fills total_us[k] / launches[k] for kinds
 * k < `kinds` (names from secure_infer_kernel_name; null past the last
 * kind) and clears the record.  Returns 0, or -1 if an event failed. */
int secure_infer_kernel_profile_enable(int on);
int secure_infer_kernel_profile_collect(double* total_us, uint64_t* launches, uint32_t kinds);
const char* secure_infer_kernel_name(uint32_t kind);

/* ------------------------------------------------- prediction scope */

/* Announce a future secure_infer_h2d_reload_layer(layer, srcs, ..., n, count,
 * codec, 0, ...) so its records are encrypted ahead of time: the host side of
 * the reference's CPU ciphertext pool (secure_infer.cpp:3264-3710, scheduled
 * by its history predictor through secure_infer_gcm_schedule_cpu_ciphertext,
 * :3526-3597).  Tickets, IVs and AADs are fixed now; a background thread
 * encrypts the records on the worker pool into a pinned buffer of a bounded
 * pool (SECURE_INFER_PREPARE_POOL_BYTES, default 256 MiB; ready entries are
 * evicted oldest first).  A later reload call with the same layer, source
 * pointers (in the same order), count and codec takes the entry, waiting for
 * it if it is still being encrypted, and copies it instead of encrypting;
 * any other reload encrypts inline as before.  The sources must not change
 * between the two calls.  Returns 0 when scheduled, 1 when not (the same
 * announcement is pending, or the pool is full), -1 on bad arguments or no
 * session. */
int secure_infer_h2d_prepare_layer(uint32_t layer, const void* const* srcs, uint32_t n, uint64_t count,
                                   const secure_infer_codec* codec);

/* secure_infer.cpp:1102-1146: end the current prediction scope.  Entries
 * announced before the call are dropped (one being encrypted is dropped when
 * it finishes); their tickets are never used. */
void secure_infer_invalidate_transfer_prefetches(void);
void secure_infer_retire_transfer_prefetches(void);

/* ------------------------------------------------------------ stats */

/* secure_infer.cpp:821-835: records reloaded from announced entries, reloads
 * that had to wait for their entry, reloads that found announced entries
 * outstanding but none matching. */
void secure_infer_get_transfer_prefetch_stats(uint64_t* ready, uint64_t* busy_fallback, uint64_t* missing_fallback);
/* secure_infer.cpp:5038-5053: scheduled, ready, hit, miss, retired, stale, failed */
void secure_infer_get_gcm_keystream_stats(uint64_t* scheduled, uint64_t* ready, uint64_t* hit, uint64_t* miss,
                                          uint64_t* retired, uint64_t* stale, uint64_t* failed);
/* worker.cpp:34-65 */
void secure_infer_get_npu_keystream_stats(uint64_t* launched, uint64_t* completed, uint64_t* failed);
void secure_infer_get_npu_keystream_pool_stats(uint64_t* slots, uint64_t* in_use);
/* secure_infer.cpp:5055 */
uint64_t secure_infer_count_ready_unconsumed_gcm_tickets(void);
/* secure_infer.cpp:6089, :6113 (profiling rows are not collected: return 0) */
int secure_infer_flush_completed_h2d_profile(void);
int secure_infer_drain_h2d_profile_after_job(void);

/* Records authenticated / rejected / retried since session init. */
void secure_infer_get_auth_stats(uint64_t* verified, uint64_t* rejected, uint64_t* retried);

/* Host-side fault injection (PIPE_GCM_TAMPER_H2D / _D2H in the reference,
 * secure_infer.cpp:6187-6251, :2454-2468): flip one byte of the nth record
 * (1-based, counted from this call) after host encryption (direction 1,
 * target 0 = ciphertext, 1 = tag) or after the device copy to the host
 * (direction 2).  nth = 0 disarms. */
void secure_infer_arm_tamper(uint32_t direction, uint64_t nth, uint32_t target);

/* ------------------------------------------------ opt-in memcpy interposer
 *
 * libsecure_infer_interpose.so (built beside this library) defines one symbol,
 * the CUDA runtime's own
 *
 *     cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t count,
 *                                 cudaMemcpyKind kind, cudaStream_t stream);
 *
 * standing in for the reference's interposed aclrtMemcpyAsync
 * (secure_infer.cpp:7729-7855).  Preloaded with SECURE_INFER_INTERPOSE=1, it
 * sends a cudaMemcpyHostToDevice copy whose source lies in a registered host
 * range to secure_infer_h2d_submit and a cudaMemcpyDeviceToHost copy into a
 * registered range to secure_infer_d2h_submit (cudaErrorInvalidValue if the
 * library refuses it); every other copy, and every copy without the variable,
 * goes to the next cudaMemcpyAsync in the lookup order.  It is not declared
 * here so that this header stays free of CUDA runtime types. */

#ifdef __cplusplus
}
#endif

#endif /* SECURE_INFER_H */
