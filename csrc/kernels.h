// Launchers for the non-GEMM sm_100a kernels (MoE dispatch/combine, norms, RoPE,
// SwiGLU, optimizer, loss). Each takes raw device pointers and a stream.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace sepx {

// Number of kernels launched by this library (incremented by every launcher).
void note_launch();
long long launch_count();

// ---------------------------------------------------------------------------------
// Expert-parallel dispatch/combine (moe_ep.cu)
// ---------------------------------------------------------------------------------
struct EpArgs {
  void* peer_base[64];  // base of every rank's symmetric region (this rank's included)
  size_t off_recv_x = 0, off_recv_e = 0, off_recv_w = 0;
  size_t off_ret_x = 0, off_ret_w = 0, off_hdr = 0;
  size_t off_recv_q = 0, off_recv_s = 0;  // e4m3 rows [W][cap][H] and 1x128 scales [W][cap][H/128]
  int W = 1, rank = 0;
  int cap = 0;  // slots per source (max tokens per rank per call)
  int k = 1;
  int H = 0;
  int T = 0;      // tokens of this rank in this call
  int phase = 0;  // header row used by this call
  uint32_t epoch = 0;
  // Optional device counter added to epoch (graph replay: a kernel in the captured
  // sequence bumps it, so every replay runs under a new epoch); null: epoch alone.
  const uint32_t* epoch_dev = nullptr;
  unsigned int* done_counter = nullptr;
  int* status = nullptr;
  unsigned long long timeout_ns = 5000000000ull;
};

// Routing of choice j of token t: dst_tk[t][j] = destination rank (-1: not sent),
// meta_tk[t][j] = value delivered with the row (local expert slot on that rank).
void ep_route_tables(const int* topk_e, const int* e2r, const int* e2l, int n, int* dst, int* meta,
                     cudaStream_t st);
// self_tok (optional): also the map slot -> token of the rows that stay on `rank`.
void ep_route_plan(const int* dst_tk, int T, int k, int W, int* slot, int* send_count, cudaStream_t st,
                   int* self_tok = nullptr, int rank = 0);
void ep_dispatch(const EpArgs& a, const void* x, const int* dst_tk, const int* meta_tk, const float* topk_w,
                 const int* slot, int* self_tok, const int* send_count, bool with_meta, cudaStream_t st,
                 bool fp8 = false);
// Receive plan in two halves so the caller can size buffers between them: count+scan
// produce group_off (group_off[G] = rows needed), permute+gather fill them.
// need / miss (optional): see recv_scan_kernel (row budgets that spare the host a wait).
void ep_recv_count_scan(const EpArgs& a, const int* dst_tk, const int* meta_tk, const float* topk_w,
                        const int* self_tok, const int* send_count, int G, int cap_rows, int* rows_from,
                        int* chunk_cnt, int* group_off, int* group_cnt, int* pad_off, cudaStream_t st,
                        int* need = nullptr, int* miss = nullptr);
void ep_recv_permute_gather(const EpArgs& a, const void* x, const int* dst_tk, const int* meta_tk,
                            const float* topk_w, const int* self_tok, const int* send_count, int G,
                            const int* rows_from, const int* chunk_cnt, const int* group_off, const int* group_cnt,
                            const int* pad_off, void* xp, float* row_w, int* row_src, int* inv_rows,
                            cudaStream_t st, bool fp8 = false);
void ep_recv_gather(const EpArgs& a, const void* x, const int* self_tok, const int* row_src,
                    const int* total_rows, const int* send_count, void* xp, int cap_rows,
                    cudaStream_t st);
// Wait for every source's header of a.phase; rows_from[src] = rows it sent.
void ep_wait_rows(const EpArgs& a, const int* send_count, int* rows_from, cudaStream_t st);
void ep_combine(const EpArgs& a, const void* y, const int* inv_rows, const float* row_w,
                const int* rows_from, bool weighted, const float* row_val, cudaStream_t st);
// World size 1: combine and source reduce in one kernel (same bits as the pair).
void ep_combine_local(const EpArgs& a, const void* y, const int* inv_rows, const float* row_w, const int* slot,
                      const int* dst_tk, bool weighted, const float* row_val, const void* residual, void* out,
                      float* val, cudaStream_t st);
void ep_source_reduce(const EpArgs& a, const int* slot, const int* dst_tk, const void* residual, void* out,
                      float* val, cudaStream_t st);

// ---------------------------------------------------------------------------------
// Speculative expert replication (speculative.cu)
// ---------------------------------------------------------------------------------
struct SpecPolicyArgs {
  const int* pred_e = nullptr;  // [T][k] predicted expert ids (negative: ignored)
  int T = 0, k = 1, E = 0;
  int S = 0;          // cache slots
  int P = 0;          // local slots before the cache (primaries + static replicas)
  int rank = 0;
  int min_count = 1;  // fewest predicted rows that make an expert worth caching
  const int* base_e2r = nullptr;  // [E] routing tables without the cache (as seen from this rank)
  const int* base_e2l = nullptr;
  const int* owner = nullptr;       // [E] primary rank of each expert
  const int* owner_slot = nullptr;  // [E] its slot on that rank
  int* slot_expert = nullptr;       // [S] cached expert per slot (-1: empty), updated
  int* slot_stamp = nullptr;        // [S] step of last use (-1: never), updated
  int* step = nullptr;              // [1] call counter, incremented
  int* e2r = nullptr;               // [E] out: routing tables with the cache
  int* e2l = nullptr;
  int* fetch_rank = nullptr;        // [S] out: rank to copy slot s from (-1: no copy)
  int* fetch_slot = nullptr;        // [S] out: slot on that rank
  long long* stats = nullptr;       // [4] accumulated: hits, fetches, predicted remote rows, of them now local
};
void spec_policy(const SpecPolicyArgs& a, cudaStream_t st);

struct SpecFetchArgs {
  const void* peer_base[64];  // every rank's symmetric weight buffer
  void* local_base = nullptr;
  int W = 1, P = 0, S = 0;
  int src_limit = 0;          // source slots must be below this (pinned slots of every rank)
  int nreg = 0;               // weight arrays per expert (e.g. gate_up and down)
  size_t reg_off[4];          // byte offset of each array in the buffer
  size_t reg_stride[4];       // bytes per expert slot of each array
  const int* fetch_rank = nullptr;
  const int* fetch_slot = nullptr;
};
void spec_fetch(const SpecFetchArgs& a, int blocks_per_slot, cudaStream_t st);

// Device timeline (trace.cu): ring[2 i] = tag, ring[2 i + 1] = %globaltimer ns.
void trace_stamp(unsigned long long* ring, unsigned int* counter, int cap, int tag, cudaStream_t st);

// All-to-all peer write bandwidth probe (p2p_bench.cu): dst[r] = rank r's buffer, each
// rank writes bytes_per_peer from src to every other rank at offset rank * bytes_per_peer.
struct P2PBenchArgs {
  uint8_t* dst[64];
  const uint8_t* src = nullptr;
  long long bytes_per_peer = 0;
  int W = 1, rank = 0, mode = 0;
  int* status = nullptr;
};
void p2p_write_bench(const P2PBenchArgs& a, int blocks, cudaStream_t st);

}  // namespace sepx
