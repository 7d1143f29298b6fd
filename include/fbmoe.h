/*
 * fbmoe.h -- C ABI of the B200-native fused FP8 block-scale DeepSeek-V3 MoE
 * operator (libfbmoe.so).  Plain pointers, sizes and a CUDA stream handle; no
 * framework types.  All tensor pointers are device pointers to contiguous
 * row-major data on the current CUDA device; every call is asynchronous on
 * `stream` and performs no host synchronisation and no device allocation.
 *
 * These entry points replace the launch chain of the reference operator
 * weichengz0616/flashinfer-bench-moe, solution/triton/main.py:
 *   fused_moe()                        main.py:2668-2774  -> fbmoe_forward
 *   fusedRoutePermuteCopyIntoWrapper   main.py:2177-2326  -> fbmoe_route (+ permute inside fbmoe_forward)
 *   gemm1_aot + actQuantWrapper        main.py:367-421, 1572-1602, 2720-2737
 *   gemm2_aot + reduceAddWrapper       main.py:748-806, 1686-1714, 2752-2771
 *   FusedMoeWorkspace                  main.py:2628-2665  -> fbmoe_workspace_size / caller-owned workspace
 *
 * Return codes: 0 on success; FBMOE_ERR_* (negative) for invalid arguments;
 * a positive value is a cudaError_t from a launch.  fbmoe_error_string()
 * describes any code.
 */
#ifndef FBMOE_H_
#define FBMOE_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FBMOE_API __attribute__((visibility("default")))
#else
#define FBMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FBMOE_HIDDEN 7168
#define FBMOE_INTERMEDIATE 2048
#define FBMOE_NUM_EXPERTS 256
#define FBMOE_TOP_K 8

#define FBMOE_OK 0
#define FBMOE_ERR_INVALID_ARG (-1)
#define FBMOE_ERR_WORKSPACE_TOO_SMALL (-2)
#define FBMOE_ERR_NULL_POINTER (-3)
#define FBMOE_ERR_MISALIGNED (-4)
#define FBMOE_ERR_DRIVER (-5)
#define FBMOE_ERR_DEVICE_STATUS (-6)
#define FBMOE_ERR_NOALLOC_LIMIT (-7)

/* Bytes of device workspace fbmoe_forward needs for T tokens and E_local local
 * experts (the reference sizes one global workspace for 15000 tokens,
 * main.py:2657; here the caller owns it and sizes it per call). */
FBMOE_API size_t fbmoe_workspace_size(int T, int E_local);

/* The fused MoE forward (reference fused_moe, main.py:2668-2774).
 *   routing_logits      fp32 [T, 256]
 *   routing_bias        bf16 [256]
 *   hidden_states       float8_e4m3fn [T, 7168]
 *   hidden_states_scale fp32 [56, T]            (1x128 block scales, transposed)
 *   gemm1_weights       float8_e4m3fn [E_local, 4096, 7168]
 *   gemm1_weights_scale fp32 [E_local, 32, 56]  (128x128 block scales)
 *   gemm2_weights       float8_e4m3fn [E_local, 7168, 2048]
 *   gemm2_weights_scale fp32 [E_local, 56, 16]
 *   out                 bf16 [T, 7168]          (written, not accumulated)
 * local_expert_offset: first global expert owned by this call (0..255);
 * E_local in {1..256}; workspace: >= fbmoe_workspace_size(T, E_local) bytes,
 * 256-byte aligned.  The result for a token is the sum over its selected
 * experts that are local. */
FBMOE_API int fbmoe_forward(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                  const float* hidden_states_scale, const void* gemm1_weights, const float* gemm1_weights_scale,
                  const void* gemm2_weights, const float* gemm2_weights_scale, int T, int E_local,
                  int local_expert_offset, float routed_scaling_factor, void* out, void* workspace,
                  size_t workspace_bytes, void* stream);

/* Same as fbmoe_forward but writes the un-rounded fp32 sum over the local experts
 * (out_f32 [T, 7168]) -- the partial that expert-parallel ranks add together
 * before the single bf16 rounding.  No reference counterpart (the reference
 * leaves combining ranks to its caller, main.py:2452-2455). */
FBMOE_API int fbmoe_forward_partial_f32(const float* routing_logits, const void* routing_bias,
                                        const void* hidden_states, const float* hidden_states_scale,
                                        const void* gemm1_weights, const float* gemm1_weights_scale,
                                        const void* gemm2_weights, const float* gemm2_weights_scale, int T,
                                        int E_local, int local_expert_offset, float routed_scaling_factor,
                                        float* out_f32, void* workspace, size_t workspace_bytes, void* stream);

/* fbmoe_forward with the reference's intermediate numerics: the SwiGLU output is
 * re-quantised to e4m3 with 1x128 scales (amax / 448, act_quant_kernel,
 * main.py:1426-1602) and GEMM2 multiplies fp8 by fp8 (gemm2_kernel,
 * main.py:433-600), each 128-K block promoted in fp32.  Applies to the prefill
 * chain (T > 64); smaller T run the decode kernel exactly as fbmoe_forward does.
 * Same arguments, workspace and errors as fbmoe_forward.  Faster GEMM2 (fp8 rate,
 * half the intermediate bytes) at the cost of the re-quantisation error, which
 * exceeds the operator's atol 1e-2 / rtol 2e-2 on a fraction of the elements:
 * not the default. */
FBMOE_API int fbmoe_forward_fp8_intermediate(const float* routing_logits, const void* routing_bias,
                                             const void* hidden_states, const float* hidden_states_scale,
                                             const void* gemm1_weights, const float* gemm1_weights_scale,
                                             const void* gemm2_weights, const float* gemm2_weights_scale, int T,
                                             int E_local, int local_expert_offset, float routed_scaling_factor,
                                             void* out, void* workspace, size_t workspace_bytes, void* stream);

/* fbmoe_forward for callers that cannot allocate device memory (no counterpart
 * in the reference).  Such callers -- a plugin host that hands over only input
 * and output pointers, a runtime whose allocator may not be called on this
 * path -- cannot supply the workspace fbmoe_forward needs, so this entry point
 * keeps it in a fixed 12 MiB device array inside the library instead.  Limits:
 * T <= 16 and E_local <= 32 (decode batches of one 32-expert shard); larger
 * sizes return FBMOE_ERR_NOALLOC_LIMIT.  The array exists on every GPU where the
 * library's device code is loaded, until the process exits.  Every call shares
 * it: calls that overlap on the GPU (e.g. on two streams) race.  The first call
 * on a device looks up the array's address (cudaGetSymbolAddress) with that
 * device current; with lazy module loading (the CUDA default) that lookup also
 * makes the driver load the library's device code there and commit the 12 MiB
 * array.  Make that first call at set-up, before any stream capture and before
 * a hot-path memory budget applies; after it no call allocates or frees device
 * memory.  Device-side errors: fbmoe_noalloc_read_status. */
FBMOE_API int fbmoe_forward_noalloc(const float* routing_logits, const void* routing_bias,
                                    const void* hidden_states, const float* hidden_states_scale,
                                    const void* gemm1_weights, const float* gemm1_weights_scale,
                                    const void* gemm2_weights, const float* gemm2_weights_scale, int T, int E_local,
                                    int local_expert_offset, float routed_scaling_factor, void* out, void* stream);

/* Device status word of the last fbmoe_forward_noalloc call on the current
 * device (no counterpart in the reference; synchronises `stream`).  The array
 * that holds the no-alloc workspace is private to the library, so this is the
 * only way its callers can see a device-side error.  Returns
 * FBMOE_ERR_DEVICE_STATUS when the word is non-zero (bits as for
 * fbmoe_read_status).  Like fbmoe_forward_noalloc, the first call on a device
 * looks up the array's address. */
FBMOE_API int fbmoe_noalloc_read_status(uint32_t* status, void* stream);

/* Offline weight pre-pack (no counterpart in the reference, which passes raw
 * weights on every call, main.py:2720-2730).  Writes W1 [E_local, 4096, 7168]
 * e4m3 with its linear half (rows 0..2047) and its silu half (rows 2048..4095)
 * interleaved in 64-row slices: packed rows [128s, 128s+64) = rows [64s, 64s+64)
 * and packed rows [128s+64, 128s+128) = rows [2048+64s, 2048+64s+64).  GEMM1 then
 * loads each operand tile as one TMA box (128 rows at decode, 256 at prefill)
 * instead of two or four.  The scales keep their layout.  `packed` must not
 * overlap `gemm1_weights`; asynchronous on `stream`. */
FBMOE_API int fbmoe_prepack_w1(const void* gemm1_weights, int E_local, void* packed, void* stream);

/* fbmoe_forward with gemm1_weights in the fbmoe_prepack_w1 layout; the result is
 * bit-identical to fbmoe_forward on the raw weights. */
FBMOE_API int fbmoe_forward_prepacked(const float* routing_logits, const void* routing_bias,
                                      const void* hidden_states, const float* hidden_states_scale,
                                      const void* gemm1_weights_packed, const float* gemm1_weights_scale,
                                      const void* gemm2_weights, const float* gemm2_weights_scale, int T,
                                      int E_local, int local_expert_offset, float routed_scaling_factor, void* out,
                                      void* workspace, size_t workspace_bytes, void* stream);

/* DeepSeek-V3 no-aux routing only (reference main.py:2522-2553 / fusedGatingKernel
 * main.py:851-1038).  topk_idx int32 [T, 8] global expert ids in canonical order
 * (descending s+bias, ascending id among equals); topk_weights fp32 [T, 8]. */
FBMOE_API int fbmoe_route(const float* routing_logits, const void* routing_bias, int T, float routed_scaling_factor,
                int32_t* topk_idx, float* topk_weights, void* stream);

/* Activation quantiser (the producer of fused_moe's hidden_states and
 * hidden_states_scale): x bf16 [T, 7168] -> q e4m3 [T, 7168] and scale fp32
 * [56, T] (transposed, as the operator takes it).  Per row and 128-column block:
 * scale = amax / 448 (1 for an all-zero block), q = e4m3(clamp(x / scale, +-448)),
 * round-to-nearest-even -- the reference's 1x128 rule, solution/triton/main.py:
 * 1476-1488 (there applied to its SwiGLU output).  x 16-byte aligned, q 8-byte;
 * values past +-448 saturate to +-448 and NaN stays NaN, as clamp then convert
 * (a NaN element converts to an e4m3 NaN of its sign and does not enter its
 * block's amax; a block holding an infinity gets scale inf).  Results equal the
 * fp32 division x / scale for every bf16 input. */
FBMOE_API int fbmoe_quantize_act(const void* x_bf16, int T, void* q_e4m3, float* scale, void* stream);

/* Byte offsets of the forward's intermediate buffers inside the workspace, for
 * inspection by tests.  `offsets` receives FBMOE_LAYOUT_FIELDS values in this
 * order: status, topk_idx, topk_w, token_rows, expert_cnt, expert_poff,
 * n_blocks, blocks, row_token, row_weight, inter, pair_out, total, row_capacity. */
#define FBMOE_LAYOUT_FIELDS 14
FBMOE_API int fbmoe_workspace_layout(int T, int E_local, int64_t* offsets);

/* Block rows (GEMM N tile) the forward picks for T tokens and E_local experts. */
FBMOE_API int fbmoe_block_rows(int T, int E_local);

/* Reads the device status word of the last forward on this workspace
 * (synchronises `stream`).  0 = clean; non-zero = a bounded wait expired inside
 * a kernel (bit 0 producer, 1 MMA, 2 epilogue, 3 converter, 5 drain, 7 peer
 * flags of an expert-parallel combine), the block list overflowed (bit 4), an f16
 * value was clamped (bit 6) or a pair row's slot was not found (bit 8). */
FBMOE_API int fbmoe_read_status(const void* workspace, uint32_t* status, void* stream);

/* Registers pinned host memory `sink` (one uint32, from cudaHostAlloc /
 * cudaMallocHost, device-accessible) as the status sink of `workspace`; NULL
 * unregisters.  The last kernel of every later forward on that workspace
 * (fbmoe_forward, fbmoe_forward_partial_f32, the expert-parallel receive) stores
 * the call's status word into the sink when it is non-zero, so a host can learn
 * of a device-side error (the bits of fbmoe_read_status) by reading the sink,
 * without synchronising.  The sink is sticky: the caller clears it.  At most 64
 * workspaces have sinks.  No reference counterpart: the reference ignores
 * launch and device status (main.py:2062-2070). */
FBMOE_API int fbmoe_set_status_sink(const void* workspace, uint32_t* sink);

/* How the decode kernel (T <= 64) was last launched: 0 not yet, 1 cooperative
 * with programmatic serialization, 2 cooperative, 3 plain programmatic launch
 * (the default).  Its CTAs wait for one another at a grid-wide arrival: every
 * launch sizes the grid to one CTA per SM after an occupancy query confirms one
 * fits; with the environment variable FBMOE_DECODE_COOPERATIVE=1 (read once per
 * process) the launch is cooperative, which also guarantees co-residency when
 * other work holds SMs, at 1-3.5 us per call on B200. */
FBMOE_API int fbmoe_decode_launch_mode(void);

/* Test hook: while `enable` is non-zero the decode kernel's grid-arrival wait
 * waits for one arrival that never comes, with a 2 ms budget, so every CTA's
 * bounded wait expires, sets status bit 2 and returns without writing its part
 * of the output.  Lets tests exercise the error path without any device fault. */
FBMOE_API int fbmoe_test_expire_grid_wait(int enable);

/* Stage timing for measurement: after fbmoe_profile_begin(n), the next n
 * forwards record CUDA events on their stream between the stages (route,
 * permute, GEMM1, GEMM2, combine).  fbmoe_profile_end synchronises those events,
 * writes the summed milliseconds per stage to stage_ms[5] and the number of
 * recorded forwards, and stops recording.  Host-side only (events, no device
 * memory); the reference has wall-clock timing only (main.py:2611-2624). */
FBMOE_API int fbmoe_profile_begin(int max_forwards);
FBMOE_API int fbmoe_profile_end(float* stage_ms, int* n_forwards);

/* ---- Expert parallelism with the combine fused into GEMM2 (NVLink peer memory).
 * Replaces the reference's single-GPU combine (reduce_add_kernel, main.py:1604-1714)
 * and the cross-rank sum of partial outputs for an expert-parallel layer sharded by
 * local_expert_offset (main.py:2558-2564).  Rank r of `world` (1..8) holds experts
 * [r*E_local, (r+1)*E_local) with E_local*world == 256 and owns output tokens
 * [r*T/world, (r+1)*T/world); T % world == 0; every rank passes the same routing
 * inputs and hidden states (replicated).  peer_recv[o] is rank o's receive buffer
 * (fbmoe_ep_recv_bytes bytes from fbmoe_ipc_alloc, mapped into this process with
 * fbmoe_ipc_open; peer_recv[rank] is this rank's own).  epoch: 1, 2, 3, ... per
 * call, the same on every rank.
 * _send: route .. GEMM2 on this rank's experts; GEMM2 stores each pair row into
 *   its owner's buffer; then releases this rank's flag on every peer.
 * _recv: waits (bounded, status bit 7) for every rank's flag of `epoch`, then
 *   out_rows_bf16 [T/world, 7168] = the sum of each owned token's 8 pair rows in
 *   slot order -- equal, bit for bit, to fbmoe_forward with all 256 experts.
 *   The status word is the one of `workspace` (fbmoe_read_status).
 * fbmoe_forward_ep = _send then _recv.  Workspace: fbmoe_ep_workspace_size. */
FBMOE_API size_t fbmoe_ep_recv_bytes(int T, int world);
FBMOE_API size_t fbmoe_ep_workspace_size(int T, int E_local);
FBMOE_API int fbmoe_forward_ep_send(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                                    const float* hidden_states_scale, const void* gemm1_weights,
                                    const float* gemm1_weights_scale, const void* gemm2_weights,
                                    const float* gemm2_weights_scale, int T, int E_local, int local_expert_offset,
                                    float routed_scaling_factor, int rank, int world, void* const* peer_recv,
                                    uint32_t epoch, void* workspace, size_t workspace_bytes, void* stream);
FBMOE_API int fbmoe_forward_ep_recv(const void* my_recv, int T, int rank, int world, uint32_t epoch,
                                    void* out_rows_bf16, void* workspace, void* stream);
FBMOE_API int fbmoe_forward_ep(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                               const float* hidden_states_scale, const void* gemm1_weights,
                               const float* gemm1_weights_scale, const void* gemm2_weights,
                               const float* gemm2_weights_scale, int T, int E_local, int local_expert_offset,
                               float routed_scaling_factor, int rank, int world, void* const* peer_recv,
                               uint32_t epoch, void* out_rows_bf16, void* workspace, size_t workspace_bytes,
                               void* stream);

/* ---- Token-dispatch expert parallelism: rank r holds only its own tokens
 * [r*T/world, (r+1)*T/world) -- routing_logits [T/world, 256], hidden_states
 * [T/world, 7168] e4m3, hidden_states_scale [56, T/world] -- and experts
 * [r*E_local, (r+1)*E_local), E_local*world == 256.  T is the global token count.
 * _send routes the rank's tokens and writes each token's top-8 into every rank's
 * dispatch buffer and its row and scales into the ranks that own one of its
 * experts (peer_dispatch[o]: rank o's fbmoe_ep_dispatch_bytes buffer), then flags
 * every peer.  _compute waits (bounded, status bit 7) for every rank's dispatch of
 * `epoch` and runs permute .. GEMM2 on this rank's experts over the global token
 * space, GEMM2 storing pair rows into the home ranks' receive buffers (peer_recv,
 * as for fbmoe_forward_ep_send), then flags them.  fbmoe_forward_ep_recv then
 * gives this rank's tokens' output rows -- equal, bit for bit, to fbmoe_forward
 * with all 256 experts on all T tokens.  fbmoe_forward_ep_dispatch = the three in
 * order.  Workspace: fbmoe_ep_workspace_size(T, E_local). */
FBMOE_API size_t fbmoe_ep_dispatch_bytes(int T, int world);
FBMOE_API int fbmoe_forward_ep_dispatch_send(const float* routing_logits, const void* routing_bias,
                                             const void* hidden_states, const float* hidden_states_scale, int T,
                                             int E_local, float routed_scaling_factor, int rank, int world,
                                             void* const* peer_dispatch, uint32_t epoch, void* workspace,
                                             size_t workspace_bytes, void* stream);
FBMOE_API int fbmoe_forward_ep_dispatch_compute(const void* gemm1_weights, const float* gemm1_weights_scale,
                                                const void* gemm2_weights, const float* gemm2_weights_scale, int T,
                                                int E_local, int rank, int world, void* my_dispatch,
                                                void* const* peer_recv, uint32_t epoch, void* workspace,
                                                size_t workspace_bytes, void* stream);
FBMOE_API int fbmoe_forward_ep_dispatch(const float* routing_logits, const void* routing_bias,
                                        const void* hidden_states, const float* hidden_states_scale,
                                        const void* gemm1_weights, const float* gemm1_weights_scale,
                                        const void* gemm2_weights, const float* gemm2_weights_scale, int T,
                                        int E_local, float routed_scaling_factor, int rank, int world,
                                        void* const* peer_dispatch, void* const* peer_recv, uint32_t epoch,
                                        void* out_rows_bf16, void* workspace, size_t workspace_bytes,
                                        void* stream);

/* Device buffers shared across processes (cudaMalloc + CUDA IPC).  A handle is
 * FBMOE_IPC_HANDLE_BYTES opaque bytes; open it in every other process of the node. */
#define FBMOE_IPC_HANDLE_BYTES 64
FBMOE_API int fbmoe_ipc_alloc(size_t bytes, void** ptr);
FBMOE_API int fbmoe_ipc_free(void* ptr);
FBMOE_API int fbmoe_ipc_handle(const void* ptr, void* handle_out);
FBMOE_API int fbmoe_ipc_open(const void* handle, void** ptr);
FBMOE_API int fbmoe_ipc_close(void* ptr);

FBMOE_API const char* fbmoe_error_string(int code);

/* Library version (major*10000 + minor*100 + patch). */
FBMOE_API int fbmoe_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FBMOE_H_ */
