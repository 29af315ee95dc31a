/*
 * exl3b200.h -- C ABI of the B200 (sm_100a) EXL3 routed-expert MoE library (libexl3b200.so).
 *
 * Plain pointers and sizes only.  Every pointer argument is a device address (or a host address the GPU can read
 * through UVA: pinned, mapped host memory) unless stated.  `stream` is a cudaStream_t (NULL = legacy default
 * stream).  All work is enqueued on `stream`; no entry point synchronises the host or allocates memory.
 * Return value: 0 = OK, 1 = invalid argument (nothing was enqueued), 2 = CUDA launch error, 3 = unsupported.
 * exl3b_last_error() gives the message of the calling thread's last failure.  Device-side errors (an index out of
 * range that a kernel skipped, a bounded wait that gave up) set bits of a device status word read by
 * exl3b_device_status().
 *
 * Each entry point names the reference interface it replaces (sybil-solutions/qwen38-flash-next-b70-offload,
 * file:line); the torch op layer in exl3b200/ops.py maps the reference's op schemas onto these calls.
 */
#ifndef EXL3B200_H
#define EXL3B200_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- misc ---------------------------------------------------------------------------------------------------- */
const char* exl3b_last_error(void);
int exl3b_abi_version(void);
/* Device status word (bits: 1 bounds, 2 bounded wait gave up, 4 bad geometry); synchronises `stream`. */
int exl3b_device_status(int* host_status, int clear, void* stream);

/* Replaces blob_bytes(H, I, K) (kernels/moe-a8/exl3_moe.a8.sycl:1551, Geom :42-54), with one K per tensor. */
int64_t exl3b_blob_bytes(int H, int I, int Kg, int Ku, int Kd);

/* ---- dequant ------------------------------------------------------------------------------------------------- */
/* Replaces exl3_reconstruct(trellis, w, n0, K, cb=mul1) (experimental/n111-victim-ring/csrc/exl3_ops.sycl:539-555,
 * ReconstructKernel kernels/moe-a8/exl3_esimd.h:869-936): tile matrix -> fp16 W_inner [rows16*16][ntiles*16] (ld ldw).
 * Row r of the tile matrix starts at words + r*row_stride_words; tiles tile0..tile0+ntiles-1 are decoded.
 * planar = 1: PLANAR4 rows (the expert blob, moe_offload.py:68-73; tile0 % 4 == 0), 0: plain checkpoint order. */
int exl3b_dequant(const void* words, int rows16, int64_t row_stride_words, int tile0, int ntiles, int K, int planar,
                  void* w_fp16, int64_t ldw, void* stream);
/* Dequantise one projection of an expert blob: proj 0 gate / 1 up -> [H][I], 2 down -> [I][H] (fp16). */
int exl3b_blob_dequant(const void* blob, int H, int I, int Kg, int Ku, int Kd, int proj, void* w_fp16, void* stream);

/* ---- router -------------------------------------------------------------------------------------------------- */
/* Replaces SGLang's TopK as consumed by Exl3XpuMoEMethod.apply (plugin/sglang_plugin.tier.py:534-535, 560):
 * logits = x . Wr^T (+ bias) with the fixed fp32 order documented in csrc/exl3b_router.cu, softmax top-k (ties to the
 * lower id), weights renormalised.  x, Wr bf16; ids int32 [T][topk]; w fp32 [T][topk]; logits fp32 [T][E] scratch. */
int exl3b_router_topk(const void* x_bf16, int64_t x_stride, const void* wr_bf16, const float* bias, int T, int H,
                      int E, int topk, int32_t* ids, float* w, float* logits, int32_t* counter, void* stream);
/* counter (may be NULL): int32 in device memory, zero before the first call, left at zero by every call; with it
 * and T <= 8 the selection runs inside the logits kernel (last block to finish), else in a second kernel.
 * Calls that share a counter must not overlap on the GPU. */

/* ---- device expert cache ------------------------------------------------------------------------------------- */
/* Replaces launch_ensure (kernels/moe-a8/exl3_moe.a8.sycl:837-1040) as called by moe_forward_cached (:1229-1261)
 * and moe_prefetch (:1194-1219), with the tier mask of moe_set_tier (:775-780) and victims of moe_set_victims
 * (:768).  Deterministic rule: masked picks logged in ascending pick order; misses in ascending expert id; victims =
 * the smallest (slot_last + 1, slot) among slots with slot_last < tick; i-th miss <-> i-th victim in slot order.
 * ids/w are rewritten in place for masked picks (ram_res != NULL).  prefetch = 1: tick not advanced, pf_slot[i]
 * receives the slots, fill_all untouched.  vict (may be NULL): [n, (old_key | -1, slot) x n]. */
int exl3b_ensure(int32_t* ids, float* w, int npairs, int layer, int E, int S, int64_t* ptrs_all, int32_t* slot_of,
                 int32_t* slot_key, int32_t* slot_last, int32_t* tick, const int64_t* host_base, int64_t slot_base,
                 int64_t blob, int64_t hstride, int64_t* fill_all, int32_t* fill_list, int max_fill, int prefetch,
                 int32_t* pf_slot, const uint8_t* ram_res, int32_t* ring, int ring_cap, const int32_t* safe,
                 int32_t* vict, void* stream);
/* Replaces the GEMV write-through fill (GateUpKernel/DownKernel `fill`, exl3_moe.a8.sycl:155-162, 207, 289) and
 * PrefetchCopyKernel (:1146-1165): copies each planned fill's blob from ptrs[e] (host tier) into its slot
 * (fill[e], or slot_base + pf_slot[i]*blob).  max_fills bounds the grid (>= fill_list[0]). */
int exl3b_fill_copy(const int32_t* fill_list, const int64_t* ptrs, const int64_t* fill, const int32_t* pf_slot,
                    int64_t slot_base, int64_t blob, int max_fills, void* stream);
/* Replaces VictimCopyKernel (exl3_moe.a8.sycl:1168-1189): victim slot -> its host address, ram_res[old] = 1. */
int exl3b_victim_copy(const int32_t* vict, const int64_t* host_base, int64_t slot_base, int64_t blob, int E,
                      int64_t hstride, uint8_t* ram_res, int max_victims, void* stream);
/* Replaces moe_set_victim_ring (experimental/n111-victim-ring/a9.patch), the victim ring variant of the write-back:
 * while set (meta != NULL), the victims of exl3b_moe_decode_cached that need a write-back are copied device to device
 * into free slots of a ring of K blob-sized slots in buf (buf_bytes >= K * blob) instead of to their host rows, and
 * ram_res is not set; the host drains the ring, flags the keys and frees the slots.  meta: int32 [4 + 2K] on the
 * device, [next search position, claim sequence, drops (ring full), K, key[K] (-1 free), seq[K]]; sel: int32 on the
 * device, one entry per victim of a call.  meta = NULL turns the ring off (direct write-back). */
int exl3b_set_victim_ring(int32_t* meta, int32_t* sel, void* buf, int64_t buf_bytes, int K);
/* Replaces the cache commit of CombineKernel (exl3_moe.a8.sycl:378-386) and moe_prefetch's table update
 * (:1212-1218): ptrs[e] = fill[e], fill[e] = 0 (or ptrs[e] = slot_base + pf_slot[i]*blob when pf_slot != NULL). */
int exl3b_commit(const int32_t* fill_list, int64_t* ptrs, int64_t* fill, const int32_t* pf_slot, int64_t slot_base,
                 int64_t blob, void* stream);

/* ---- copy-engine prefetch ------------------------------------------------------------------------------------ */
/* Replaces moe_prefetch_plan (kernels/moe-a8/exl3_moe.a8.sycl:1127-1142), the plan mode of launch_ensure
 * (:898-1036): commits landed plans (as exl3b_cepf_commit); then, unless this layer's previous plan is still in
 * flight, claims up to max_fill (<= 16) LRU slots for the experts of ids that are not in VRAM, exactly as
 * exl3b_ensure's prefetch mode does (tick not advanced), pins them (slot_last = INT_MAX), records them in pend
 * (int32 [n_layers][35]: n, seq, T, (expert, slot) x 16) and publishes [seq, n, T, layer, (expert, slot) x n] to the
 * layer's record of plans (pinned host memory, int32 [n_layers][4 + 2E]), seq written last behind a system-scope
 * fence.  plan_seq: int32 [n_layers] device counters.  The table keeps pointing at the host copies until the commit. */
int exl3b_cepf_plan(const int32_t* ids, int n, int layer, int E, int S, int64_t* ptrs_all, int32_t* slot_of,
                    int32_t* slot_key, int32_t* slot_last, int32_t* tick, const int64_t* host_base, int64_t slot_base,
                    int64_t blob, int64_t hstride, int32_t* pf_list, int32_t* pf_slot, int max_fill, int32_t* plans,
                    int32_t* plan_seq, int32_t* pend, const int32_t* done_seq, int n_layers, void* stream);
/* Replaces the pend / done_seq commit at the head of launch_ensure (:874-896): every layer whose done_seq (int32
 * [n_layers], written by the worker's copy stream) reached its pending seq gets its planned ptrs_all entries pointed
 * at their slots and the slots unpinned (slot_last = the plan's tick). */
int exl3b_cepf_commit(int32_t* pend, const int32_t* done_seq, int n_layers, int E, int S, int64_t* ptrs_all,
                      int32_t* slot_last, int64_t slot_base, int64_t blob, void* stream);
/* Replaces moe_prefetch_worker_start / moe_prefetch_worker_stop (:1048-1124): one host thread per process that turns
 * each newly published plan into cudaMemcpyAsync copies (host_base[layer] + expert * hstride -> slot) on copy_stream
 * followed by a kernel writing done_seq[layer] = seq on the same stream.  host_base: host array of n_layers addresses.
 * stop handles the plans already published, waits for copy_stream, writes counts[0] = plans, counts[1] = copies, and
 * returns non-zero when a copy failed (that plan then stays in flight and its experts are read from host). */
int exl3b_cepf_worker_start(const int32_t* plans, int n_layers, int E, int S, const int64_t* host_base,
                            int64_t slot_base, int64_t blob, int64_t hstride, int32_t* done_seq, int device,
                            void* copy_stream);
int exl3b_cepf_worker_stop(int64_t* counts);
int exl3b_cepf_worker_running(void);

/* ---- routed MoE, decode (few tokens) ------------------------------------------------------------------------- */
/* Replaces moe_forward_impl's GEMV path (exl3_moe.a8.sycl:1263-1314: GateUpKernel :121-260, DownKernel :264-368,
 * CombineKernel :371-395) for M tokens (any M; intended for M <= 64): out[m] = sum_k w[m,k] * expert(ids[m,k])(x[m]).
 * x fp16 (x_bf16 = 0) or bf16 [M][x_stride]; ids int32 / w fp32 [M][topk] contiguous; ptrs int64 [E] blob
 * addresses; kinfo (NULL = uniform K) int32 [E] per-expert Kg | Ku << 4 | Kd << 8; out [M][out_stride] with
 * out_bf16 = 0 fp16, 1 bf16, 2 fp32 (the un-rounded layer output).
 * flags bit 0: skip picks whose weight is exactly 0 (tier-masked picks; the output is unchanged).
 * workspace: >= exl3b_moe_decode_workspace(M, topk, H, I) bytes, 256-byte aligned, owned by the caller. */
int64_t exl3b_moe_decode_workspace(int M, int topk, int H, int I);
int exl3b_moe_decode(const void* x, int64_t x_stride, int x_bf16, const int32_t* ids, const float* w, int M, int topk,
                     const int64_t* ptrs, const int32_t* kinfo, int H, int I, int K, int E, void* out,
                     int64_t out_stride, int out_bf16, void* workspace, int64_t ws_bytes, int flags, void* stream);
/* Replaces moe_forward_cached (kernels/moe-a8/exl3_moe.a8.sycl:1229-1261): the device cache step of exl3b_ensure
 * (same state tensors, same deterministic rule, tier mask and victims), then the decode above on the layer's table
 * ptrs_all + layer*E.  Cache fills are read from their host address during the call and copied into their slots; the
 * table is repointed (commit) by the last block of the call.  ids / w are rewritten in place for masked picks.
 * vict (may be NULL) enables the victim write-back (VictimCopyKernel) with vict_ram_res flags. */
int exl3b_moe_decode_cached(const void* x, int64_t x_stride, int x_bf16, int32_t* ids, float* w, int M, int topk,
                            int layer, int64_t* ptrs_all, int32_t* slot_of, int32_t* slot_key, int32_t* slot_last,
                            int32_t* tick, const int64_t* host_base, int64_t slot_base, int64_t blob, int64_t hstride,
                            int64_t* fill_all, int32_t* fill_list, int max_fill, int S, const uint8_t* ram_res,
                            int32_t* ring, int ring_cap, const int32_t* safe, int32_t* vict, uint8_t* vict_ram_res,
                            int H, int I, int K, int E, void* out, int64_t out_stride, int out_bf16, void* workspace,
                            int64_t ws_bytes, int flags, void* stream);
/* Router + cached decode in one call (no reference counterpart: the reference plugin takes the picks from SGLang's
 * TopK, plugin/sglang_plugin.tier.py:534-535, and calls moe_forward_cached with them, exl3_moe.a8.sycl:1229-1261).
 * The same results as exl3b_router_topk (x_bf16, wr_bf16, bias -> ids, w, logits) followed by exl3b_moe_decode_cached
 * on them: ids / w are written (and rewritten in place for masked picks) as those two calls would.  For small batches
 * (M <= 8, M topk <= 32) the router kernel writes only the logits and the decode kernels select the picks from them
 * (one grid completion and the router's last-block arrival fewer per call); larger batches make the two calls.
 * logits: [M][E] fp32; counter: the router's fused-selection counter (may be NULL), used for larger batches. */
int exl3b_moe_decode_cached_routed(const void* x_bf16, int64_t x_stride, const void* wr_bf16, const float* bias,
                                   float* logits, int32_t* ids, float* w, int M, int topk, int layer, int64_t* ptrs_all,
                                   int32_t* slot_of, int32_t* slot_key, int32_t* slot_last, int32_t* tick,
                                   const int64_t* host_base, int64_t slot_base, int64_t blob, int64_t hstride,
                                   int64_t* fill_all, int32_t* fill_list, int max_fill, int S, const uint8_t* ram_res,
                                   int32_t* ring, int ring_cap, const int32_t* safe, int32_t* vict,
                                   uint8_t* vict_ram_res, int H, int I, int K, int E, void* out, int64_t out_stride,
                                   int out_bf16, void* workspace, int64_t ws_bytes, int flags, int32_t* counter,
                                   void* stream);
/* Profiling hook (no reference counterpart; the reference times graph replays from the host,
 * plugin/sglang_plugin.tier.py:1036-1087): cudaEvent_t handles recorded by exl3b_moe_decode before its route
 * prep, gate-up and down kernels and after down, and by exl3b_moe_prefill before align, before the gate-up GEMM,
 * before the down GEMM and after the combine.  NULL disables a slot.  Process-global, off by default. */
int exl3b_set_profile_events(void* before_route, void* before_gateup, void* before_down, void* after_down);

/* ---- routing tables ------------------------------------------------------------------------------------------ */
/* Replaces launch_align / moe_align (kernels/moe-a8/exl3_moe.a8.sycl:639-680, 1317-1325; buffers as make_route
 * :744-757): picks bucketed by expert with a stable counting sort (ascending pick index inside an expert).
 * ib int32 = [act_expert A | act_start A | act_cnt A | act_pstart A | n_act 1 | pair_tok P | pair_of P | 16 |
 * blk_a mxb | n_blk 1], pair_w fp32 [P]; A = min(P, E), mxb = ceil(P / pad) + A.
 * scratch: >= exl3b_align_scratch(P, E) bytes of device memory. */
int64_t exl3b_align_scratch(int P, int E);
int exl3b_align(const int32_t* ids, const float* w, int P, int topk, int E, int pad, int32_t* ib, float* pair_w, int A,
                int mxb, void* scratch, int64_t scratch_bytes, void* stream);

/* No counterpart in the reference.  exl3b_moe_decode for callers that cannot allocate device memory: the same
 * kernels and arguments without workspace / ws_bytes; the scratch is a fixed 8 MiB device array of the library
 * (exl3b_moe_decode_workspace(M, topk, H, I) must be <= 8 MiB: up to 85 tokens at top-10 with H = 2048, I = 768; larger
 * calls return EXL3B_EINVAL).  The first call on each device looks the array's address up, so make it before any
 * stream capture on that device.  Nothing has to be zeroed by the caller.  One scratch per device: calls that overlap
 * on one device race; order them on one stream or with events. */
int exl3b_moe_decode_noalloc(const void* x, int64_t x_stride, int x_bf16, const int32_t* ids, const float* w, int M,
                             int topk, const int64_t* ptrs, const int32_t* kinfo, int H, int I, int K, int E, void* out,
                             int64_t out_stride, int out_bf16, int flags, void* stream);

/* Config-5 shared expert: replaces the model's shared_expert_gate (a bf16 Linear(H -> 1) + sigmoid around the
 * shared expert, whose three linears go through exl3xpu_C.linear, experimental/n111-victim-ring/csrc/exl3_ops.sycl:
 * 651-757).  Weight = 1 / (1 + expf(-dot(x[t], g))) with the router's dot-product arithmetic; writes the extended
 * routing ids_out / w_out [T][topk + 1] = the routed picks, then (shared_id, weight).  The shared expert's blob (the
 * routed layout, its own K per tensor) is entry shared_id of the pointer table given to the MoE layer, so it runs as
 * one more pick per token and enters the combine after the routed picks. */
int exl3b_shared_gate(const void* x_bf16, int64_t x_stride, const void* g_bf16, int T, int H, const int32_t* ids,
                      const float* w, int topk, int shared_id, int32_t* ids_out, float* w_out, void* stream);

/* ---- expert-parallel prefill (configs[3]; the reference's moe_prefill, exl3_moe.a8.sycl:792-828, runs on one GPU:
 * this is its extension over G GPUs of one node, around NCCL all-to-all exchanges done by the host).
 * Experts are sharded contiguously, rank d owning ids [d E/G, (d+1) E/G).  exl3b_ep_plan: for the T local tokens'
 * routing ids / w [T][topk] (id -1 = no pick), bits [T] scratch, counts [G] / offs [G+1] (int64) rows per
 * destination and their offsets, pos [T][G] = send row of (t, d) or -1 (destination-major, ascending t), and per
 * send row (at most T G): send_src (source token), send_ids / send_w [topk] (the destination's local expert ids,
 * -1 for picks owned by other ranks).  exl3b_ep_pack: send_x[row] = x[send_src[row]] (16-bit rows).
 * exl3b_ep_combine: out[t] = sum over d ascending of part[pos[t][d]] (fp32 partial sums returned by the
 * destinations), out_kind 0 fp16, 1 bf16, 2 fp32. */
int exl3b_ep_plan(const int32_t* ids, const float* w, int T, int topk, int E, int G, uint32_t* bits, int64_t* counts,
                  int64_t* offs, int32_t* pos, int32_t* send_src, int32_t* send_ids, float* send_w, void* stream);
int exl3b_ep_pack(const void* x, int64_t x_stride, int H, const int32_t* send_src, int n_rows, void* send_x,
                  void* stream);
int exl3b_ep_combine(const float* part, const int32_t* pos, int T, int G, int H, void* out, int64_t out_stride,
                     int out_kind, void* stream);

/* The exchange EPPrefill runs: one all-to-all of send records each way with equal splits (every rank passes the same
 * cap >= its T), so the host never reads the counts.  exl3b_ep_record_bytes: bytes of one record, 2 H + 8 topk rounded
 * up to 16.  exl3b_ep_dispatch: send [G cap] records, destination d's block rows [d cap, (d + 1) cap): its first
 * counts[d] rows the local tokens that pick d (ascending t), each record the token's row of x (H 16-bit values), then
 * its topk ids as d's local expert ids (int32, -1 for picks owned elsewhere), then their weights (fp32, 0 for those);
 * the block's other rows have ids -1 and weights 0 (and an unwritten row of x), so the destination can run its MoE
 * layer over all G cap received rows.  counts int64 [2 G + 1] (rows per destination, then scratch), pos [T][G] = the
 * send row of (t, d) or -1, bits [T] and src [G cap] scratch.  exl3b_ep_combine_h: exl3b_ep_combine over fp16 partial
 * sums (the destinations return [G cap][H] fp16, summed here in fp32 in ascending rank order). */
int64_t exl3b_ep_record_bytes(int H, int topk);
int exl3b_ep_dispatch(const void* x, int64_t x_stride, const int32_t* ids, const float* w, int T, int topk, int E, int G,
                      int H, int cap, uint32_t* bits, int64_t* counts, int32_t* pos, int32_t* src, void* send,
                      void* stream);
int exl3b_ep_combine_h(const void* part, const int32_t* pos, int T, int G, int H, void* out, int64_t out_stride,
                       int out_kind, void* stream);

/* Replaces moe_prefill (kernels/moe-a8/exl3_moe.a8.sycl:792-828 with GateUpDpasKernel :422-545, DownDpasKernel
 * :548-635 and CombineKernel :371-395), the path moe_forward takes for M >= prefill_min_m (:1263-1314): the routed-MoE
 * layer for many tokens as grouped tensor-core GEMMs (tcgen05, fp16 operands, fp32 accumulate in TMEM).  Arguments as
 * exl3b_moe_decode; H % 256 == 0, I % 128 == 0.  Every pick's weighted output is stored fp16 and the combine sums
 * those in fp32 in pick order, as the reference's prefill does.
 * workspace: >= exl3b_moe_prefill_workspace(M, topk, H, I, E) bytes, 1024-byte aligned, owned by the caller. */
int64_t exl3b_moe_prefill_workspace(int M, int topk, int H, int I, int E);
int exl3b_moe_prefill(const void* x, int64_t x_stride, int x_bf16, const int32_t* ids, const float* w, int M, int topk,
                      const int64_t* ptrs, const int32_t* kinfo, int H, int I, int K, int E, void* out,
                      int64_t out_stride, int out_bf16, void* workspace, int64_t ws_bytes, int flags, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* EXL3B200_H */
