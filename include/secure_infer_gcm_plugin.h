/*
 * secure_infer_gcm_plugin.h -- device crypto plugin ABI ("GHASH_LIBRARY").
 *
 * CUDA (sm_100a) edition of the entry points the reference data plane loads
 * from its device crypto plugin with dlopen/dlsym
 * (secure_infer/native/secure_infer.cpp:335-421).  Names, argument order and
 * argument meaning follow the reference declarations
 * (secure_infer/native/secure_infer.h:396-457) and wrappers
 * (secure_infer/native/kernels/aicpu/launcher.asc:23-524).
 *
 * Conventions for every function below:
 *   - `stream` is a cudaStream_t (nullptr = the CUDA legacy default stream);
 *     all other pointers are device pointers; work is ordered on `stream`.
 *   - returns 0 when the work was enqueued, -1 for null/zero arguments or
 *     an unsupported size; the call never waits for the device.
 *   - iv_word0..3 are big-endian packs of the 16 IV bytes; word 3 is the
 *     first 32-bit block counter (2 for a GCM payload; J0 uses 1).
 *   - verify paths write plaintext, or zeros when the tag does not match,
 *     and store uint32 1/0 to `status_output`.
 *   - all arguments are captured at enqueue time: nothing the caller passes
 *     (including the host pointer arrays of the *_batch_do calls) needs to
 *     outlive the call.
 * The device X25519 key agreement (launcher.asc:23-33) is not exported: the
 * reference treats that symbol as optional and session setup is outside the
 * transfer path.
 */
#ifndef SECURE_INFER_GCM_PLUGIN_H
#define SECURE_INFER_GCM_PLUGIN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SECURE_INFER_KEYSTREAM_BATCH_MAX 32u     /* ghash_shared.h:62 */
#define SECURE_INFER_VERIFY_XOR_BATCH_MAX 4u     /* ghash_shared.h:147 */

/* ghash_do flags (ghash_shared.h:24-28) */
#define SECURE_INFER_GHASH_FINALIZE_TAG (1u << 0)
#define SECURE_INFER_GHASH_VERIFY_TAG (1u << 1)
#define SECURE_INFER_GHASH_XOR_ON_SUCCESS (1u << 2)

/* GHASH over AAD || input || len; FINALIZE xors tag_mask, VERIFY compares with
 * expected_tag, XOR_ON_SUCCESS writes (input ^ keystream) or zeros.
 * Replaces launcher.asc:75-114 / ghash.aicpu:978-1046. */
int secure_infer_aicpu_ghash_do(void* stream, void* input, void* hash_subkey, void* output, void* aad,
                                void* tag_mask, void* expected_tag, void* keystream, void* plaintext_output,
                                void* status_output, uint64_t input_bytes, uint64_t aad_bytes, uint32_t flags);

/* Zero `data` unless *status == 1.  launcher.asc:116-132 / ghash.aicpu:1051-1068. */
int secure_infer_aicpu_auth_gate_do(void* stream, void* data, void* status, uint64_t bytes);

/* Device half of the experimental X25519 + BLAKE2b session key agreement
 * (launcher.asc:23-33 / key_agreement.aicpu): from the host's 32-byte X25519
 * public value and 32-byte challenge, writes the device public value (32 B),
 * the 16-byte session key (it stays in device memory) and the 32-byte proof
 * BLAKE2b(key = session key, challenge); *status (int32) = 0 when done.  The
 * device secret is hashed from on-chip timers (B200 has no entropy source). */
int secure_infer_aicpu_key_agreement_do(void* stream, void* host_public, void* challenge, void* device_key,
                                        void* device_public, void* proof, void* status);

/* AES-128-CTR XOR of `bytes` bytes.  launcher.asc:134-155 / ghash.aicpu:517-535. */
int secure_infer_aicpu_aes_ctr_do(void* stream, void* input, void* key, void* output, uint64_t bytes,
                                  uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2, uint32_t iv_word3);

/* AES-128-CTR keystream only.  launcher.asc:160-179 / ghash.aicpu:537-554. */
int secure_infer_aicpu_keystream_do(void* stream, void* key, void* output, uint64_t bytes, uint32_t iv_word0,
                                    uint32_t iv_word1, uint32_t iv_word2, uint32_t iv_word3);

/* Up to 32 independent (IV, output) keystreams under one key; iv_words is a
 * host array [count][4].  launcher.asc:184-210 / ghash.aicpu:559-582. */
int secure_infer_aicpu_keystream_batch_do(void* stream, void* key, void* const* outputs, const uint32_t* iv_words,
                                          uint64_t bytes, uint32_t count);

/* Fused tag check + CTR decrypt (keystream computed in the kernel).
 * launcher.asc:214-275 / ghash.aicpu:594-651. */
int secure_infer_aicpu_gcm_decrypt_verify_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                             void* expected_tag, void* plaintext_output, void* status_output,
                                             uint64_t bytes, uint32_t iv_word0, uint32_t iv_word1,
                                             uint32_t iv_word2, uint32_t iv_word3);
int secure_infer_aicpu_gcm_decrypt_verify_aad_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                                 void* expected_tag, void* plaintext_output, void* status_output,
                                                 uint64_t bytes, uint32_t iv_word0, uint32_t iv_word1,
                                                 uint32_t iv_word2, uint32_t iv_word3, void* aad,
                                                 uint64_t aad_bytes);

/* CTR encrypt + tag = GHASH(AAD || C || len) ^ E_K(J0).
 * launcher.asc:279-308 / ghash.aicpu:656-699. */
int secure_infer_aicpu_gcm_encrypt_tag_do(void* stream, void* plaintext, void* key, void* hash_subkey,
                                          void* ciphertext_output, void* tag_output, uint64_t bytes,
                                          uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2,
                                          uint32_t iv_word3, void* aad, uint64_t aad_bytes);

/* Tag check + XOR with a precomputed keystream.
 * launcher.asc:312-376 / ghash.aicpu:705-773. */
int secure_infer_aicpu_gcm_verify_xor_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                         void* expected_tag, void* keystream, void* plaintext_output,
                                         void* status_output, uint64_t bytes, uint32_t iv_word0, uint32_t iv_word1,
                                         uint32_t iv_word2, uint32_t iv_word3);
int secure_infer_aicpu_gcm_verify_xor_aad_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                             void* expected_tag, void* keystream, void* plaintext_output,
                                             void* status_output, uint64_t bytes, uint32_t iv_word0,
                                             uint32_t iv_word1, uint32_t iv_word2, uint32_t iv_word3, void* aad,
                                             uint64_t aad_bytes);

/* Tag check only.  launcher.asc:378-435 / ghash.aicpu:780-827. */
int secure_infer_aicpu_gcm_verify_only_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                          void* expected_tag, void* status_output, uint64_t bytes,
                                          uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2,
                                          uint32_t iv_word3);
int secure_infer_aicpu_gcm_verify_only_aad_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                              void* expected_tag, void* status_output, uint64_t bytes,
                                              uint32_t iv_word0, uint32_t iv_word1, uint32_t iv_word2,
                                              uint32_t iv_word3, void* aad, uint64_t aad_bytes);

/* Up to 4 independent records (own IV, tag, keystream, output, status) in one
 * launch; pointer arrays and iv_words [count][4] are host arrays.
 * launcher.asc:440-486 / ghash.aicpu:834-940. */
int secure_infer_aicpu_gcm_verify_xor_batch_do(void* stream, void* key, void* hash_subkey, void* const* ciphertexts,
                                               void* const* expected_tags, void* const* keystreams,
                                               void* const* plaintext_outputs, void* const* status_outputs,
                                               void* const* aads, uint64_t bytes, uint64_t aad_bytes,
                                               const uint32_t* iv_words, uint32_t count);

/* Profiling control: XOR only, status forced to 1, NO authentication.
 * launcher.asc:495-524 / ghash.aicpu:948-976. */
int secure_infer_aicpu_gcm_xor_only_do(void* stream, void* ciphertext, void* key, void* hash_subkey,
                                       void* expected_tag, void* keystream, void* plaintext_output,
                                       void* status_output, uint64_t bytes, uint32_t iv_word0, uint32_t iv_word1,
                                       uint32_t iv_word2, uint32_t iv_word3);

/* Allocation-free variant of secure_infer_aicpu_gcm_decrypt_verify_aad_do.
 * No counterpart in the reference.  For callers that cannot call cudaMalloc
 * (code inside an allocator or memory budget it does not own, or a path that
 * must never pay for a device allocation): the entry points above allocate a
 * per-stream scratch area on first use, this one keeps its scratch (key
 * schedule, segment partials, arrival counter; about 1 MiB, held by every
 * GPU that loads the library until exit) in a fixed device array.  Same
 * arguments, meaning and results; returns -2 with a message on stderr when
 * bytes > 16 MiB or aad_bytes > 4096.  Every call looks up the array's
 * address on the current device (so it stays valid after cudaDeviceReset);
 * the first call on a device may load the module, so make it before any
 * stream capture.  Every call shares
 * the array: calls whose work overlaps on the GPU race and must be serialised
 * by the caller. */
int secure_infer_aicpu_gcm_decrypt_verify_aad_noalloc_do(void* stream, void* ciphertext, void* key,
                                                         void* hash_subkey, void* expected_tag,
                                                         void* plaintext_output, void* status_output,
                                                         uint64_t bytes, uint32_t iv_word0, uint32_t iv_word1,
                                                         uint32_t iv_word2, uint32_t iv_word3, void* aad,
                                                         uint64_t aad_bytes);

#ifdef __cplusplus
}
#endif

#endif /* SECURE_INFER_GCM_PLUGIN_H */
