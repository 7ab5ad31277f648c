// Attention metadata of one forward step, built on the device.
//
// Device side of the reference's ModelRunner.prepare_seqs
// (src/engine/model_runner.py:174-233).  Per sequence b the host uploads only
//   start[b]  = min(num_cached_tokens, len - 1)
//   lq[b]     = num_scheduled_tokens          (end = start + lq)
//   nblk[b]   = length of its block table (0: no table, as in warm-up)
// and the -1-padded block tables; this kernel expands them per token:
//   cu_seqlens_q = prefix sums of lq, cu_seqlens_k = prefix sums of end,
//   context_lens = end, positions of the tokens [start, end) of each
//   sequence, and slot(p) = block_table[p / page] * page + p % page for the
//   tokens of sequences that have a table (the reference leaves the others
//   out of slot_mapping, model_runner.py:198-199).
// One CTA per sequence; each CTA sums the lengths of the sequences before it
// (B is at most a few thousand, so the redundant prefix sums cost less than a
// second launch).
#pragma once
#include "common.cuh"

namespace b200 {

struct MetaArgs {
  const int* start;         // [B]
  const int* lq;            // [B]
  const int* nblk;          // [B]
  const int* block_tables;  // [B][bt_stride]
  int bt_stride, B, page;
  long long* positions;     // [T]
  int* slot_mapping;        // [tokens of sequences with a table]
  int* cu_q;                // [B + 1]
  int* cu_k;                // [B + 1]
  int* context_lens;        // [B]
  unsigned* err;
};

__global__ void __launch_bounds__(256) step_metadata_kernel(const MetaArgs a) {
  griddep_wait();
  griddep_launch_dependents();
  __shared__ long long s_red[3][8];
  const int b = blockIdx.x;
  long long sq = 0, sk = 0, ss = 0;
  for (int i = threadIdx.x; i < b; i += blockDim.x) {
    const int l = a.lq[i];
    sq += l;
    sk += a.start[i] + l;
    ss += a.nblk[i] > 0 ? l : 0;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
    sk += __shfl_xor_sync(0xffffffffu, sk, o);
    ss += __shfl_xor_sync(0xffffffffu, ss, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    s_red[0][warp] = sq;
    s_red[1][warp] = sk;
    s_red[2][warp] = ss;
  }
  __syncthreads();
  sq = sk = ss = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    sq += s_red[0][w];
    sk += s_red[1][w];
    ss += s_red[2][w];
  }
  const int start = a.start[b], lq = a.lq[b], nb = a.nblk[b];
  if (threadIdx.x == 0) {
    if (b == 0) {
      a.cu_q[0] = 0;
      a.cu_k[0] = 0;
    }
    a.cu_q[b + 1] = (int)(sq + lq);
    a.cu_k[b + 1] = (int)(sk + start + lq);
    a.context_lens[b] = start + lq;
  }
  const int* bt = a.block_tables + (size_t)b * a.bt_stride;
  for (int j = threadIdx.x; j < lq; j += blockDim.x) {
    const int p = start + j;
    a.positions[sq + j] = p;
    if (nb > 0) {
      const int col = p / a.page;
      int slot = -1;
      if (col < nb) {
        const int blk = bt[col];
        if (blk >= 0) slot = blk * a.page + (p - col * a.page);
      }
      if (slot < 0) raise_error(a.err, ERR_BAD_INDEX);
      a.slot_mapping[ss + j] = slot;
    }
  }
}

}  // namespace b200
