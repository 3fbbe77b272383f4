// Allocation-free C entry point for MLA paged decode attention.
//
// This entry point has no counterpart in the reference: it is an addition of
// this library for callers that cannot allocate device memory themselves.
//
// Who needs it: code that must not call cudaMalloc (or any allocator) on the
// decode path, for example a host runtime written in another language that
// links this .so directly and hands over only its own tensors, a process that
// runs under a memory budget fixed at start-up, or a real-time serving loop
// where an allocation could block or fail in the middle of a step. Such a
// caller passes its inputs and output; the split-KV partial results, which the
// regular entry point keeps in freshly allocated scratch tensors, live here in
// a fixed file-scope device array instead.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// Largest scratch the entry point can use: 16 MiB per GPU that loads the
// library, held until the process exits. A call needs
//   batch * splits * heads * (kv_lora + 1) * 4 bytes   (kv_lora = 512)
// when splits > 1; splits == 1 needs no scratch at all.
#define SP_MLA_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

// Return codes (0 = launched). Positive values are cudaError_t codes.
#define SP_NOALLOC_OK 0
#define SP_NOALLOC_BAD_ARGUMENT (-1)
#define SP_NOALLOC_SCRATCH_TOO_SMALL (-2)
#define SP_NOALLOC_SETUP_FAILED (-3)

// MLA decode attention over a paged latent cache (kv_lora 512 + rope 64,
// 64-token blocks), exactly the computation of the package's mla_decode op:
//   q            [batch, heads, 576] bf16 (device)
//   cache        [num_slots, 576] bf16 (device, one layer)
//   block_table  [batch, max_blocks] int32 (device)
//   context_lens [batch] int32 (device)
//   out          [batch, heads, 512] bf16 (device)
//   stream       cudaStream_t to launch on (0 = legacy default stream)
//
// The first call on a device (with that device current) resolves the device
// address of the scratch array once; make that first call before any stream
// capture begins. Every call on a device shares the same scratch array, which
// keeps the previous call's contents: two calls whose kernels overlap on the
// GPU (different streams without ordering between them) race on it, so order
// them on one stream or with events. The status word that the kernel's bounded
// waits write is cleared on the stream before each launch.
// Nothing is allocated: no cudaMalloc / cudaFree and no allocating library
// routine is called.
__attribute__((visibility("default"))) int sp_mla_decode_noalloc(
    const void* q, const void* cache, long long num_slots, const int* block_table, int max_blocks,
    const int* context_lens, void* out, int batch, int heads, int splits, float scale, void* stream);

// Reads (and clears) the status word of the calls made on the current device:
// 0 = no bounded wait ran out. It first waits for `stream` (the stream the calls
// were launched on; 0 = legacy default stream) to finish, so a call launched on a
// non-blocking stream has written its status before it is read. Blocks the host;
// returns a negative value on failure.
__attribute__((visibility("default"))) int sp_mla_decode_noalloc_status(void* stream);

#ifdef __cplusplus
}
#endif
