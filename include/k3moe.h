/* k3moe — B200 (sm_100a) routed-MoE layer of Kimi-K3: the C ABI.
 *
 * Every entry takes caller-owned device buffers, plain pointers and sizes,
 * and a CUDA stream; it enqueues work and returns 0, or a negative K3MOE_E*
 * code for bad arguments or a launch failure.  Nothing here allocates device
 * memory on the hot path; the layer entry carves its intermediates out of a
 * caller-provided workspace (k3moe_layer_workspace_size).  Device-side
 * failures (a routing-table entry out of range, a bounded wait that ran out)
 * are written to the error words inside the workspace and read back with
 * k3moe_read_error after the stream is synchronised; no kernel traps.
 *
 * Layouts (HBM):
 *   activations x        bf16 [T, ldx]
 *   router logits S      f32  [T, lds], E_total experts wide
 *   expert weights       MXFP4: E2M1 two a byte (element 2i in the low nibble
 *                        of byte i).  W13 of expert e is [gate rows 0..I-1 ;
 *                        up rows I..2I-1] x H, W2 is H x I, experts back to
 *                        back (W13 [E*2I, H], W2 [E*H, I]), stored TILE-MAJOR:
 *                        128 x 128-element tiles, tile (r/128, k/128) at index
 *                        (r/128)*(K/128) + k/128, each tile row-major (8 KB);
 *                        byte of element (r, k): tile*8192 + (r%128)*64 + (k%128)/2.
 *   weight scales        UE8M0 per 32 along K, 128x4-tiled over the
 *                        flattened rows (byte of row r, group kb at
 *                        ((r/128)*(K/128) + kb/4)*512 + (r%32)*16 + (r%128/32)*4 + kb%4):
 *                        scale atom t belongs to data tile t.
 *   GEMM activations     MXFP8 E4M3 in the same tile-major layout (tile*16384
 *                        + (r%128)*128 + k%128) with scales tiled as above;
 *                        the plain quantiser entry writes row-major q.
 *   routing tables       the reference's format (docs/k3-kernel-abi.md K14,
 *                        source/k3_moe_prefill.cu:12-35): cta_batch, cta_limit,
 *                        num_non_exiting, total_padded, route_map, exp2perm.
 */
#ifndef K3MOE_H
#define K3MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* k3moe_stream_t; /* a cudaStream_t */

enum {
  K3MOE_OK = 0,
  K3MOE_EINVAL = -1,     /* an argument is out of the supported range */
  K3MOE_ENOSPACE = -2,   /* workspace smaller than k3moe_layer_workspace_size */
  K3MOE_EDRIVER = -3,    /* the CUDA driver entry for tensor maps is unavailable */
  K3MOE_ETMAP = -4,      /* a tensor map could not be encoded (alignment / size) */
  K3MOE_ELAUNCH = -5,    /* a kernel launch failed (cudaGetLastError) */
  K3MOE_EDEVICE = -6,    /* k3moe_read_error: the device reported a failure */
  K3MOE_ELIMIT = -7      /* a size beyond the fixed scratch of k3moe_route_tables_noalloc */
};

/* Version of this ABI. */
int k3moe_abi_version(void);

/* ---------------------------------------------------------------- router top-k
 * sig = 1/(1+expf(-S)), key = sig + bias; the K largest keys, ties to the
 * smaller expert, in descending order; wts = sig / (sum of the K sig + 1e-20)
 * * rs, the sum an xor butterfly over the K picks.  K a power of two <= 16,
 * E_total <= 1024.  Bit-identical to the reference's router top-k.
 * Replaces: kern_k3g_router_topk (source/k3_prefill_glue.cu:504-557),
 *   phase 1 of kern_k3g_moe_route (source/k3_moe_route.cu:117-221, 372-385). */
int k3moe_route_topk(const float* S, int lds, const float* bias, const void* rs_bf16, int T, int E_total, int K,
                     int32_t* idx, float* wts, k3moe_stream_t stream);

/* ---------------------------------------------------------------- the router GEMM
 * S[t, e] = sum_h x[t, h] * W[e, h]: bf16 x bf16 -> f32 on the tensor cores (x [T, ldx], W [E, ldw], S
 * [T, lds]), the logits the top-k reads.  H a multiple of 64, E of 16; ldx, ldw multiples of 8 and lds of 4;
 * pointers 16-byte aligned.  err: the device error words (a bounded wait that ran out), or null.
 * Replaces: the router projection gemm(L + "router", normed, w_router, router_partial, EXPERTS, H)
 *   (scripts/gen_stage.py:1130), bound to extern:cublas_bf16_tn_f32 (gen_stage.py:244-247). */
int k3moe_router_gemm(const void* x_bf16, int ldx, const void* w_bf16, int ldw, int T, int E, int H, float* S, int lds,
                      uint32_t* err, k3moe_stream_t stream);

/* ---------------------------------------------------------------- routing tables
 * Over R rows with K ids each (global expert indices), the local experts being
 * [first, first + E): counts[e], the CTA tables of `tile`-row tiles,
 * meta[0] = num_non_exiting, meta[1] = total_padded, meta[2] = first permuted
 * row of the shared expert (or -1), route_map[perm] = row (padding rows 0),
 * exp2perm[r*K + k] = perm or -1 (foreign expert).  With shared = 1 a further
 * local expert E takes every row.  Within an expert the rows are in row
 * order, so the tables are the same bytes on every run.  The K ids of one row
 * must be distinct (as top-k ids are); to rank repeated ids (e.g. destination
 * ranks), pass them one a row (K = 1).  tile = 1 plans positions only (no CTA
 * tables are written).
 * scratch: k3moe_route_scratch_bytes(R, E, shared) bytes.  E + shared <= 2048.
 * Replaces: kern_k3_moe_route_count / _tables / _scatter
 *   (source/k3_moe_prefill.cu:97-204), phase 2 of kern_k3g_moe_route
 *   (source/k3_moe_route.cu:457-519), FlashInfer's routing offsets. */
size_t k3moe_route_scratch_bytes(int R, int E, int shared);
int k3moe_route_tables(const int32_t* idx, int R, int K, int first, int E, int shared, int tile, void* scratch,
                       int32_t* counts, int32_t* cta_batch, int32_t* cta_limit, int32_t* meta, int32_t* route_map,
                       int32_t* exp2perm, k3moe_stream_t stream);

/* Capacity bounds of the tables: CTAs <= E + shared + ceil((R*K + shared*R) / tile). */
int k3moe_max_ctas(int R, int K, int E, int shared, int tile);

/* k3moe_route_tables for callers that cannot allocate device memory (a host
 * runtime that owns all device buffers and binds a fixed list to each call, or
 * a latency-critical loop that cannot afford cudaMalloc's possible device-wide
 * synchronisation): the same tables, with the scratch taken from an array
 * compiled into the library instead of a caller buffer; nothing is allocated.
 * Limits: R <= K3MOE_NOALLOC_MAX_ROWS and E + shared <= K3MOE_NOALLOC_MAX_EXPERTS,
 * else K3MOE_ELIMIT.  The array (513 KB) is one per device and shared by every
 * call: calls that overlap on the GPU race on it.  The first call on a device
 * looks the array up (make it before any stream capture).
 * No counterpart in the reference: it has no allocation-free variant. */
#define K3MOE_NOALLOC_MAX_ROWS 16384
#define K3MOE_NOALLOC_MAX_EXPERTS 1025
int k3moe_route_tables_noalloc(const int32_t* idx, int R, int K, int first, int E, int shared, int tile,
                               int32_t* counts, int32_t* cta_batch, int32_t* cta_limit, int32_t* meta,
                               int32_t* route_map, int32_t* exp2perm, k3moe_stream_t stream);

/* ---------------------------------------------------------------- MXFP8 quantisation
 * Per 32 elements along a row: e = ceil(log2(amax/448)) (0 when amax is 0),
 * clamped to [-127, 127]; sf = e + 127 (UE8M0); q = E4M3(x * 2^-e), round to
 * nearest even, saturating.  cols a multiple of 256.
 * tiled_sf = 0: sf linear [rows, cols/32]     (kern_k3_moe_quant, source/k3_moe_prefill.cu:66-95)
 * tiled_sf = 1: sf in the 128x4-tiled layout  (kern_k3_mxfp8_quant, source/k3_mxfp8.cu:20-54) */
int k3moe_quant_mxfp8(const void* x_bf16, int ldx, int rows, int cols, uint8_t* q, uint8_t* sf, int tiled_sf,
                      k3moe_stream_t stream);

/* The same quantisation written to every permuted row a row is routed to:
 * q_perm [cap, cols], sf_perm tiled over permuted rows.  (The reference
 * quantises unpermuted and gathers inside FC1; this build permutes here.) */
int k3moe_quant_permute(const void* x_bf16, int ldx, int R, int cols, int K, const int32_t* exp2perm,
                        const int32_t* meta, uint8_t* q_perm, uint8_t* sf_perm, k3moe_stream_t stream);

/* ---------------------------------------------------------------- grouped GEMMs
 * FC1: for every token tile c and 128 features f of its expert e:
 *   g = W13_e[f] . x, u = W13_e[I + f] . x (block-scaled, f32 accumulate),
 *   h = silu(g) * u, requantised to MXFP8 (the rule above) into
 *   fc1_q [cap, I] / fc1_sf (tiled over permuted rows).
 * FC2: fc2 [cap, H] bf16 = W2_e . fc1 over each tile's rows.
 * Tables from k3moe_route_tables (tile 128).  H, I multiples of 256; fc1_q
 * and fc2_bf16 32-byte aligned (K3MOE_EINVAL otherwise); err: the device
 * error words (2 x u32).
 * Replaces: the FC1 / FC2 batched GEMMs (kernels.toml:1-9; arguments
 *   scripts/k3_moe_bmm.py:131-134, 167-169; docs/k3-kernel-abi.md:535-565). */
int k3moe_fc1(const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* q_perm, const uint8_t* sf_perm,
              const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, uint8_t* fc1_q,
              uint8_t* fc1_sf, int H, int I, int n_experts, int cap_rows, int max_ctas, uint32_t* err,
              k3moe_stream_t stream);
int k3moe_fc2(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
              const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, void* fc2_bf16, int H, int I,
              int n_experts, int cap_rows, int max_ctas, uint32_t* err, k3moe_stream_t stream);

/* FC1 with the gate chosen: K3MOE_ACT_SWIGLU h = silu(g) * u (k3moe_fc1), or
 * K3MOE_ACT_SITU, K3's h = 4 tanh(g/4) sigmoid(g) * 25 tanh(u/25)
 * (docs/k3-kernel-abi.md:73; harness/k3/ref.h:97-101; the FC1 cubin's
 * siTuGlu with alpha 4, beta 25: scripts/k3_moe_bmm.py:16-20). */
enum { K3MOE_ACT_SWIGLU = 0, K3MOE_ACT_SITU = 1 };
int k3moe_fc1_act(const uint8_t* w13, const uint8_t* w13_sf, const uint8_t* q_perm, const uint8_t* sf_perm,
                  const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, uint8_t* fc1_q,
                  uint8_t* fc1_sf, int H, int I, int n_experts, int cap_rows, int max_ctas, uint32_t* err,
                  int activation, k3moe_stream_t stream);

/* The two TMA descriptors (128 bytes each: the weights', then the activations') that the module entries
 * kern_k3_moe_fc1 / kern_k3_moe_fc2 of k3moe_module.cubin read through their `maps` argument, encoded for buffers at fixed addresses and copied to maps_dev (K3MOE_GEMM_MAPS_BYTES of
 * device memory, 64-byte aligned): a load-time call, once the buffers are placed; it synchronises `stream`.  mode 0: FC1 over w = W13 [n_experts*2I, H/2]
 * and act = q_perm [cap_rows, H]; mode 1: FC2 over w = W2 [n_experts*H, I/2] and act = fc1_q [cap_rows, I].
 * The module entries take the reference ops' parameter lists (scripts/k3_moe_bmm.py:131-134, 167-169) and
 * replace the trtllm_bmm launches of scripts/k3_moe_bmm.py:112-113, whose 17,472-byte parameter block carries
 * its own descriptors (docs/k3-kernel-abi.md:549-565). */
#define K3MOE_GEMM_THREADS 384        /* block of kern_k3_moe_fc1 / kern_k3_moe_fc2 */
#define K3MOE_GEMM_SMEM_BYTES 204032  /* their dynamic shared memory */
#define K3MOE_GEMM_MAPS_BYTES 256     /* their descriptor buffer */
int k3moe_gemm_tensor_maps(int mode, const uint8_t* w, const uint8_t* act, int n_experts, int H, int I, int cap_rows,
                           void* maps_dev, k3moe_stream_t stream);

/* FC2 over the output columns [col0, col0 + ncols) only (multiples of 256), stored at
 * out_bf16 + out_rows[r] * ldo (out_rows null: row r), with at most grid_cap persistent
 * blocks (0: one an SM; fewer leave SMs to a collective running beside it). */
int k3moe_fc2_cols(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
                   const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, const int32_t* out_rows,
                   void* out_bf16, int ldo, int col0, int ncols, int H, int I, int n_experts, int cap_rows,
                   int max_ctas, int grid_cap, uint32_t* err, k3moe_stream_t stream);

/* FC2 storing permuted row r at row out_rows[r] of fc2_bf16 (the expert-parallel
 * layer passes route_map, so rows come out in the order they were received). */
int k3moe_fc2_to_rows(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
                      const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, const int32_t* out_rows,
                      void* fc2_bf16, int H, int I, int n_experts, int cap_rows, int max_ctas, uint32_t* err,
                      k3moe_stream_t stream);

/* ---------------------------------------------------------------- expert parallelism
 * Tokens are owned by their rank; each rank holds E_local experts.  Two wire
 * formats: one row a pick (the fixed-block decode mode), k3moe_ep_row_stride(H)
 * bytes: E4M3 [H] | UE8M0 [H/32] | int32 local expert id; and one row a token
 * and destination rank (below, k3moe_ep_pack_pairs).
 * No counterpart in the reference for the MoE (its decode EP replicates the
 * batch and all-reduces: roofline/decode.md:164-166; k3_ar_fused.cu:916). */
int k3moe_ep_row_stride(int H);
/* Quantise row t of x once and write it to send slots send_pos[t*K + k] (>= 0)
 * with id idx % E_local; with send_pos null, to slot t with id fixed_eid. */
int k3moe_ep_pack(const void* x_bf16, int ldx, int T, int H, int K, const int32_t* idx, const int32_t* send_pos,
                  int E_local, int fixed_eid, uint8_t* dst, int stride, k3moe_stream_t stream);
/* ids[i] = the local expert id of packed row i. */
int k3moe_ep_ids(const uint8_t* rows, int stride, int R, int H, int32_t* ids, k3moe_stream_t stream);
/* Packed row i -> permuted row perm[i] (>= 0) of the GEMM operand (tile-major q, tiled scales). */
int k3moe_ep_unpack(const uint8_t* rows, int stride, int R, int H, const int32_t* perm, uint8_t* q_perm,
                    uint8_t* sf_perm, k3moe_stream_t stream);
/* Per-destination rows (the counts-exchange dispatch): a token travels once to
 * each rank holding any of its picks, as E4M3 [H] | UE8M0 [H/32] | int16 [K]
 * local expert ids of its picks there (pick order, -1 after), stride
 * k3moe_ep_pair_row_stride(H, K).  The receiver routes a row to all its
 * experts and returns FC2's results one row a pick, so k3moe_combine_ep is
 * unchanged.  W (ranks) <= 32. */
int k3moe_ep_pair_row_stride(int H, int K);
/* pair_ids[t*W + d] = d when token t has a pick on rank d (dest[t*K + k] == d), else -1. */
int k3moe_ep_pairs(const int32_t* dest, int T, int K, int W, int32_t* pair_ids, k3moe_stream_t stream);
/* Quantise row t once; write it to slot pair_pos[t*W + d] (>= 0) of every rank d it goes to, headed by
 * lid[t*K + k] for its picks with dest[t*K + k] == d; with pair_pos null, to slot t headed by fixed_eid. */
int k3moe_ep_pack_pairs(const void* x_bf16, int ldx, int T, int H, int K, const int32_t* dest, const int32_t* lid,
                        const int32_t* pair_pos, int W, int fixed_eid, uint8_t* dst, int stride,
                        k3moe_stream_t stream);
/* ids[i*K + j] = the j-th local expert id of per-destination row i (-1 none). */
int k3moe_ep_ids_k(const uint8_t* rows, int stride, int R, int H, int K, int32_t* ids, k3moe_stream_t stream);
/* Per-destination row i -> permuted rows perm[i*K + j] (>= 0) of the GEMM operand. */
int k3moe_ep_unpack_k(const uint8_t* rows, int stride, int R, int H, int K, const int32_t* perm, uint8_t* q_perm,
                      uint8_t* sf_perm, k3moe_stream_t stream);
/* out_rows[perm[i*K + j]] = the (i, j) pair's number among the valid pairs in (i, j) order: the return row of
 * FC2's result (k3moe_fc2_to_rows). */
int k3moe_ep_return_rows(const int32_t* perm, int R, int K, int32_t* out_rows, k3moe_stream_t stream);
/* out[t] = bf16( sum_k fma(wts[t,k], back[pos[t,k]], acc) (pos >= 0, k in order) + shared[t] ):
 * the combine over rows returned by the combine all-to-all (shared_bf16 may be null). */
int k3moe_combine_ep(const void* back_bf16, const int32_t* pos, const float* wts, const void* shared_bf16,
                     int ld_shared, void* out_bf16, int ldo, int T, int K, int cols, k3moe_stream_t stream);

/* k3moe_combine_ep over rows that come as column chunks of chunk_cols columns (cols a multiple of it):
 * chunk j of returned row p at back + j * back_chunk_stride + p * back_ld elements, of shared row t at
 * shared + j * shared_chunk_stride + t * ld_shared (the expert-parallel layer returns FC2's results one
 * column chunk at a time, each all-to-all overlapping the next chunk's FC2). */
int k3moe_combine_ep_chunked(const void* back_bf16, long long back_chunk_stride, int back_ld, const int32_t* pos,
                             const float* wts, const void* shared_bf16, long long shared_chunk_stride, int ld_shared,
                             void* out_bf16, int ldo, int T, int K, int cols, int chunk_cols, k3moe_stream_t stream);

/* ---------------------------------------------------------------- expert parallelism over peer memory
 * The same exchange without the two all-to-all passes: the pack kernel stores each row straight into the
 * destination rank's receive buffer, and FC2's epilogue stores each result row straight into the owner's
 * return buffer, over NVLink through CUDA IPC mappings; then a flag a (source rank, phase) tells the receiver
 * that a source's stores are complete.  The owner's combine (k3moe_combine_ep) reads only local memory: the
 * combine is folded into the collective's receive side.  W <= 16 ranks.
 * Replaces the combine fused with the collective of the reference's decode step (kern_k3_ar_finalize_rms,
 * source/k3_ar_fused.cu:916, a Lamport all-reduce over peer memory; its spin waits end in __trap, these end
 * in an error word). */
/* k3moe_ep_pack_pairs with rank d's slot p at row_base[d] + p * stride (row_base: host array of W device
 * addresses, 16-byte aligned; a peer's receive buffer shifted by the slots of lower ranks). */
int k3moe_ep_pack_pairs_to(const void* x_bf16, int ldx, int T, int H, int K, const int32_t* dest, const int32_t* lid,
                           const int32_t* pair_pos, int W, const uint64_t* row_base, int stride,
                           k3moe_stream_t stream);
/* row_ptrs[perm[i*K + j]] = the address of the (i, j) pair's result row: with q = out_rows[perm] in block s
 * ([block_start[s], block_start[s+1]), s < nblocks), block_base[s] + (q - block_start[s]) * row_bytes
 * (host arrays; bases 32-byte aligned).  A q in no block is recorded in err (site 0xB00) and sent to `sink`
 * (a local row of row_bytes). */
int k3moe_ep_row_ptrs(const int32_t* perm, int R, int K, const int32_t* out_rows, int nblocks,
                      const uint64_t* block_base, const int64_t* block_start, int64_t row_bytes, void* sink,
                      uint64_t* row_ptrs, uint32_t* err, k3moe_stream_t stream);
/* FC2 storing permuted row r at the device address row_ptrs[r] (a row of H bf16 columns, 32-byte aligned,
 * in this GPU's memory or a peer's). */
int k3moe_fc2_to_ptrs(const uint8_t* w2, const uint8_t* w2_sf, const uint8_t* fc1_q, const uint8_t* fc1_sf,
                      const int32_t* cta_batch, const int32_t* cta_limit, const int32_t* meta, const uint64_t* row_ptrs,
                      int H, int I, int n_experts, int cap_rows, int max_ctas, uint32_t* err, k3moe_stream_t stream);
/* After this stream's earlier stores: epoch into slot slot0 + me of every other rank's flag array
 * (flag_bases: host array of W device addresses of u32 flag arrays, peers' through IPC). */
int k3moe_ep_signal(const uint64_t* flag_bases, int W, int me, int slot0, uint32_t epoch, k3moe_stream_t stream);
/* Wait on the device until flags[s] >= epoch (serial-number order) for every s < W but `skip`, at most
 * budget_ns: a source still late then is recorded in err (K3MOE_EDEVICE from k3moe_read_error: bit 0, site
 * 0xA00 + s) and the wait returns; later work on the stream runs (the caller checks err). */
int k3moe_ep_wait(const uint32_t* flags, int W, int skip, uint32_t epoch, uint64_t budget_ns, uint32_t* err,
                  k3moe_stream_t stream);
/* CUDA IPC of a buffer inside any device allocation: a 64-byte handle of the allocation holding dev_ptr and
 * dev_ptr's offset in it; import maps a peer's handle into this process (peer access enabled) and returns
 * the buffer's address; release unmaps it. */
int k3moe_ipc_export(const void* dev_ptr, void* handle64, uint64_t* offset);
int k3moe_ipc_import(const void* handle64, uint64_t offset, void** dev_ptr);
int k3moe_ipc_release(void* dev_ptr, uint64_t offset);

/* ---------------------------------------------------------------- combine
 * out[t] = bf16( sum over k = 0..K-1 with exp2perm >= 0 of fma(wts, fc2[p], acc)
 * in f32, k in order, then + fc2[meta[2] + t] when meta and meta[2] >= 0 );
 * rows t in [T, out_rows) are zero.  cols a multiple of 8.
 * Replaces: kern_k3_moe_finalize (source/k3_moe_prefill.cu:206-234). */
int k3moe_combine(const void* fc2_bf16, const int32_t* exp2perm, const float* wts, const int32_t* meta, void* out_bf16,
                  int ldo, int T, int out_rows, int K, int cols, k3moe_stream_t stream);

/* ---------------------------------------------------------------- weights
 * fp32 [rows, K] -> MXFP4 (OCP MX: scale 2^(floor(log2 amax) - 2), RNE to
 * E2M1, saturate at 6); packed [rows, K/2], scales tiled (see top).
 * No reference counterpart: the reference consumes pre-quantised checkpoints. */
int k3moe_quant_mxfp4(const float* w, long long rows, int K, uint8_t* packed, uint8_t* sf, k3moe_stream_t stream);
/* A checkpoint's MXFP4 expert weights into the layout above, on the device (once, at load): packed_rows
 * [experts * rows_per_expert, K/2] E2M1 (element 2i in the low nibble) and scale_rows
 * [experts * rows_per_expert, K/32] UE8M0, both row-major, experts back to back, as the checkpoint's
 * `weight_packed` / `weight_scale` tensors are bound; -> packed (tile-major) and sf (128x4-tiled).
 * gated = 1 for FC1, whose checkpoint rows come as [w3 (up); w1 (gate)]: the halves are swapped into
 * [gate; up].  rows_per_expert and K multiples of 128; packed pointers 16-byte, scale pointers 4-byte aligned.
 * Replaces: the load-time kern_k3_moe_w_shuffle / kern_k3_moe_sf_shuffle (source/k3_moe_prefill.cu:237-259;
 *   scripts/k3_moe_bmm.py:176-184; bound at scripts/gen_stage.py:681-702), which lay the same bytes out
 *   for the TRT-LLM-gen GEMMs; the module entries kern_k3_moe_w_tiles / kern_k3_moe_sf_tiles take
 *   their parameter lists. */
int k3moe_import_mxfp4(const uint8_t* packed_rows, const uint8_t* scale_rows, int experts, int rows_per_expert,
                       int K, int gated, uint8_t* packed, uint8_t* sf, k3moe_stream_t stream);
/* Synthetic weights of stream `seed` (rows [row0, row0+rows)), quantised as above. */
int k3moe_synth_mxfp4(uint64_t seed, long long row0, long long rows, int K, float sd, uint8_t* packed, uint8_t* sf,
                      k3moe_stream_t stream);

/* ---------------------------------------------------------------- the layer
 * One routed-MoE layer on the experts this GPU holds: top-k -> tables ->
 * MXFP8 permute -> FC1 -> FC2 -> combine (+ the shared expert, stored as
 * local expert E of the weight tensors, applied to every row with weight 1).
 * Replaces the chain of scripts/k3_moe_bmm.py:150-170 (route, fc1, fc2,
 * finalize) for one rank holding every expert. */
typedef struct k3moe_layer_args {
  int T;              /* rows this call routes */
  int H, I;           /* hidden, expert intermediate (multiples of 256) */
  int E;              /* routed experts (= router width) */
  int K;              /* top-k */
  int shared;         /* 1: expert E of the weights is the always-on shared expert */
  const float* S;     /* router logits f32 [T, lds] */
  int lds;
  const float* bias;  /* f32 [E] */
  const void* rs;     /* bf16 [1] routed scale */
  const void* x;      /* bf16 [T, ldx] */
  int ldx;
  const uint8_t* w13; const uint8_t* w13_sf;  /* [E + shared, 2I, H/2] */
  const uint8_t* w2;  const uint8_t* w2_sf;   /* [E + shared, H, I/2] */
  void* out;          /* bf16 [T, ldo] */
  int ldo;
  int activation;     /* FC1 gate: K3MOE_ACT_SWIGLU (0) or K3MOE_ACT_SITU (1) */
} k3moe_layer_args;

size_t k3moe_layer_workspace_size(int T, int H, int I, int E, int K, int shared);
int k3moe_layer_forward(const k3moe_layer_args* a, void* workspace, size_t ws_bytes, k3moe_stream_t stream);
/* The same call recording CUDA events (cudaEvent_t, may be null) on `stream`
 * before each stage and after the last: [0] top-k, [1] tables, [2] MXFP8
 * permute, [3] FC1, [4] FC2, [5] combine, [6] end (n_events <= 7 used). */
int k3moe_layer_forward_events(const k3moe_layer_args* a, void* workspace, size_t ws_bytes, k3moe_stream_t stream,
                               void* const* events, int n_events);

/* Intermediates of the last k3moe_layer_forward inside `workspace`, for
 * inspection and tests: byte offsets of idx, wts, counts, cta_batch,
 * cta_limit, meta, route_map, exp2perm, q_perm, sf_perm, fc1_q, fc1_sf, fc2,
 * err (14 entries). */
int k3moe_layer_workspace_offsets(int T, int H, int I, int E, int K, int shared, size_t* offsets14);

/* ---------------------------------------------------------------- the expert-parallel layer, device-resident
 * One rank's part of an expert-parallel MoE layer over peer memory (NVLink / NVSwitch), as one call that
 * enqueues the whole step and never synchronises with the host: top-k -> the sender's plans -> MXFP8 pack
 * stored straight into the destinations' receive buffers -> a flag exchange -> tables -> FC1 -> FC2 storing
 * each result row into its owner's return buffer -> a flag exchange -> the owner's combine.  Every rank's
 * receive buffer has a fixed region a source rank (max_tokens rows), so a rank needs no other rank's counts
 * before it sends; the whole step can be captured in a CUDA graph.  The output is the bytes of
 * k3moe_layer_forward over all ranks' experts (same arithmetic, same summation order).
 * Each rank holds E / world routed experts (owner: host int32 [E], the rank of each expert, E / world each, a
 * rank's experts in increasing id order being its local experts 0, 1, ...; NULL: contiguous blocks) and, with
 * shared, a replica of the shared expert as local expert E / world of its weight tensors.
 * Set-up, on every rank: allocate k3moe_ep_peer_bytes (zeroed, 256-byte aligned) and
 * k3moe_ep_workspace_bytes; export the peer buffer (k3moe_ipc_export), exchange the handles, import the
 * peers' (k3moe_ipc_import); k3moe_ep_create; then a host barrier across the ranks before any rank's first
 * k3moe_ep_forward (create clears this rank's flags).  Every rank calls k3moe_ep_forward the same number of
 * times.  A peer that stays late past wait_budget_ns is recorded in the error words (k3moe_ep_errors; bit 0,
 * site 0xA00 + 0x10 * phase + rank) and the step completes with what arrived; nothing traps.  world <= 16.
 * No counterpart in the reference for the MoE (its decode EP replicates the batch and all-reduces,
 * roofline/decode.md:164-166; its fused all-reduce + finalize kern_k3_ar_finalize_rms,
 * source/k3_ar_fused.cu:916, is the combine-with-collective this step's FC2 epilogue stores replace). */
typedef struct k3moe_ep_config {
  int world, rank;
  int H, I;                 /* multiples of 256 */
  int E, K;                 /* routed experts in all (E % world == 0, E <= 1024), top-k (a power of 2, <= 16) */
  int shared;               /* 1: local expert E / world is the always-on shared expert */
  int max_tokens;           /* tokens a rank per call (T <= max_tokens) */
  int activation;           /* FC1 gate: K3MOE_ACT_SWIGLU (0) or K3MOE_ACT_SITU (1) */
  uint64_t wait_budget_ns;  /* bound of each flag wait (0: 5 s) */
} k3moe_ep_config;
typedef struct k3moe_ep k3moe_ep;

size_t k3moe_ep_peer_bytes(const k3moe_ep_config* c);
size_t k3moe_ep_workspace_bytes(const k3moe_ep_config* c);
/* peer_bases: host array [world], every rank's peer buffer as mapped in this process ([rank] = peer_buffer).
 * Weights: this rank's experts, tile-major as above. */
int k3moe_ep_create(const k3moe_ep_config* c, const int32_t* owner, const uint8_t* w13, const uint8_t* w13_sf,
                    const uint8_t* w2, const uint8_t* w2_sf, void* peer_buffer, const uint64_t* peer_bases,
                    void* workspace, size_t ws_bytes, k3moe_stream_t stream, k3moe_ep** out);
/* One step over this rank's T tokens: S f32 [T, lds] router logits (E wide), bias f32 [E], rs bf16 [1],
 * x bf16 [T, ldx], out bf16 [T, ldo]. */
int k3moe_ep_forward(k3moe_ep* ep, const float* S, int lds, const float* bias, const void* rs_bf16,
                     const void* x_bf16, int ldx, int T, void* out_bf16, int ldo, k3moe_stream_t stream);
/* The same call recording CUDA events (may be null) on `stream`: [0] start, [1] after top-k and the plans,
 * [2] after the dispatch (pack + exchange), [3] after tables + unpack, [4] after FC1, [5] after FC2, [6] after
 * the combine exchange, [7] after the combine (n_events <= 8 used). */
int k3moe_ep_forward_events(k3moe_ep* ep, const float* S, int lds, const float* bias, const void* rs_bf16,
                            const void* x_bf16, int ldx, int T, void* out_bf16, int ldo, k3moe_stream_t stream,
                            void* const* events, int n_events);
/* The step's device error words (two u32, for k3moe_read_error); the rows received in the last step
 * (counts, W + 1 u32 device words: per source rank, then this rank's shared rows). */
uint32_t* k3moe_ep_errors(k3moe_ep* ep);
const uint32_t* k3moe_ep_counts(k3moe_ep* ep);
/* The last step's routing tables on this rank: rows routed to each local expert (E / world + shared int32
 * device words) and meta (num_non_exiting, total_padded, ...: 4 int32 device words). */
const int32_t* k3moe_ep_expert_rows(k3moe_ep* ep);
const int32_t* k3moe_ep_meta(k3moe_ep* ep);
/* Frees the host object only (the caller owns every buffer). */
void k3moe_ep_destroy(k3moe_ep* ep);

/* Tracing: with a device buffer of 32 zeroed u64 set, every later FC1 / FC2
 * launch of this process adds per-role SM cycle counters into it (FC1 at
 * [0..15], FC2 at [16..31]): [0] producer cycles, [1] producer cycles waiting
 * for a free stage, [2] MMA-issuer cycles, [3] waiting for a loaded stage,
 * [4] waiting for the accumulator to be drained, [5] epilogue cycles (one
 * warp), [6] epilogue waiting for an accumulator, [7] work units.  Summed over
 * blocks.  Null turns tracing off (the default). */
int k3moe_set_trace(uint64_t* counters);

/* Read (and clear, when clear != 0) the two device error words at `err`:
 * returns 0 when both are zero, else K3MOE_EDEVICE with the words in out2.
 * Synchronises `stream`. */
int k3moe_read_error(uint32_t* err, uint32_t* out2, int clear, k3moe_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* K3MOE_H */
