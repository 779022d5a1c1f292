// Small HBM-bound kernels around the tensor-core GEMMs: forward finalisation, the
// cross-shard combine, split-K reduction, f32 -> bf16 conversion, and the response-token
// compaction (warp-ballot scan + row gather) with its scatter back to the slot layout.
#pragma once

#include "lp_ptx.cuh"

namespace lpk {

// Merge the per-unit (max2, sum) partials of every vocab group (and column half) of one
// shard. A partial of a half that saw only vocabulary padding is (-inf, 0) and adds 0.
//   stats[0][t] = max (natural units), stats[1][t] = sum exp(z - max),
//   stats[2][t] = owned target logit or 0;  logp[t] = stats[2] - (max + log sum)
__global__ void fwd_finalize_kernel(const float2* __restrict__ part, int n_groups, int T,
                                    const float* __restrict__ tgt_ws, const int32_t* __restrict__ y, long long v_off,
                                    long long Vs, float* __restrict__ stats, float* __restrict__ logp) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float m = -INFINITY;
  for (int g = 0; g < n_groups; ++g) m = fmaxf(m, part[(size_t)g * T + t].x);
  float s = 0.f;
  for (int g = 0; g < n_groups; ++g) {
    const float2 p = part[(size_t)g * T + t];
    s += p.y * exp2f(p.x - m);
  }
  const long long local = (long long)y[t] - v_off;
  const bool owned = local >= 0 && local < Vs;
  const float tgt = owned ? tgt_ws[t] : 0.f;
  const float mx = m * kLn2;
  stats[t] = mx;
  stats[(size_t)T + t] = s;
  stats[(size_t)2 * T + t] = tgt;
  if (logp != nullptr) logp[t] = tgt - (mx + logf(s));
}

// fwd_finalize_kernel for few rows with many partials (small T: one block per row, each
// thread folds a strided subset of the partials, then the block reduces). Same outputs.
__global__ void fwd_finalize_rows_kernel(const float2* __restrict__ part, int n_groups, int T,
                                         const float* __restrict__ tgt_ws, const int32_t* __restrict__ y,
                                         long long v_off, long long Vs, float* __restrict__ stats,
                                         float* __restrict__ logp) {
  __shared__ float2 warp_ms[32];
  const int t = blockIdx.x;
  float m = -INFINITY, s = 0.f;
  for (int g = threadIdx.x; g < n_groups; g += blockDim.x) {
    const float2 p = part[(size_t)g * T + t];
    if (p.x == -INFINITY) continue;
    const float nm = fmaxf(m, p.x);
    s = s * exp2f(m - nm) + p.y * exp2f(p.x - nm);
    m = nm;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float om = __shfl_down_sync(0xffffffffu, m, off);
    const float os = __shfl_down_sync(0xffffffffu, s, off);
    const float nm = fmaxf(m, om);
    if (nm != -INFINITY) {
      s = (m == -INFINITY ? 0.f : s * exp2f(m - nm)) + (om == -INFINITY ? 0.f : os * exp2f(om - nm));
      m = nm;
    }
  }
  if ((threadIdx.x & 31) == 0) warp_ms[threadIdx.x >> 5] = make_float2(m, s);
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
    const float2 o = warp_ms[w];
    const float nm = fmaxf(m, o.x);
    if (nm == -INFINITY) continue;
    s = (m == -INFINITY ? 0.f : s * exp2f(m - nm)) + (o.x == -INFINITY ? 0.f : o.y * exp2f(o.x - nm));
    m = nm;
  }
  const long long local = (long long)y[t] - v_off;
  const bool owned = local >= 0 && local < Vs;
  const float tgt = owned ? tgt_ws[t] : 0.f;
  const float mx = m * kLn2;
  stats[t] = mx;
  stats[(size_t)T + t] = s;
  stats[(size_t)2 * T + t] = tgt;
  if (logp != nullptr) logp[t] = tgt - (mx + logf(s));
}

// Per-row (max, sum, owned target) of this shard from the forward GEMM's partials.
__device__ __forceinline__ float3 shard_triple(const float2* __restrict__ part, int n_groups, int T, int t,
                                               const float* __restrict__ tgt_ws, const int32_t* __restrict__ y,
                                               long long v_off, long long Vs) {
  float m = -INFINITY;
  for (int g = 0; g < n_groups; ++g) m = fmaxf(m, part[(size_t)g * T + t].x);
  float s = 0.f;
  for (int g = 0; g < n_groups; ++g) {
    const float2 p = part[(size_t)g * T + t];
    s += p.y * exp2f(p.x - m);
  }
  const long long local = (long long)y[t] - v_off;
  const bool owned = local >= 0 && local < Vs;
  return make_float3(m * kLn2, s, owned ? tgt_ws[t] : 0.f);
}

// The forward's finalize on one rank of a vocabulary mesh, fused with the exchange of the
// per-shard triples over NVLink (the pmax / psum of losses.py:219,243-245):
//   1. every thread merges its rows' partials into this shard's (max, sum, owned target)
//      (or reads them from `pre`, merged by fwd_finalize_rows_kernel when T is small) and
//      stores them, as one 16-byte multimem store, into slot `rank` of every rank's
//      copy of the exchange buffer [world][ld] (f32x4);
//   2. the last block of this launch to finish step 1 (an arrival counter in this GPU's
//      memory) adds 1 to the exchange counter in every copy (release at system scope);
//   3. every block waits (bounded) until its local copy of the counter reaches `target`
//      (epoch * world: all ranks have stored), then merges the `world` triples of its rows
//      exactly as combine_kernel does: logp = tgt - m - log s, norm = (m, s).
// All blocks of the grid must be resident at once (the host keeps the grid at or below the
// SM count), since a block only waits after its own stores. A block whose wait runs out
// records DEV_TIMEOUT_PEER and writes NaN to its rows of logp / norm.
__global__ void fwd_finalize_mesh_kernel(const float2* __restrict__ part, int n_groups, int T,
                                         const float* __restrict__ tgt_ws, const int32_t* __restrict__ y,
                                         long long v_off, long long Vs, float4* xch_mc, const float4* xch_local,
                                         long long ld, unsigned* cnt_mc, const unsigned* cnt_local, unsigned* arrivals,
                                         unsigned target, int rank, int world, unsigned long long limit_ns,
                                         const float* __restrict__ pre, float* __restrict__ logp,
                                         float* __restrict__ norm) {
  __shared__ int s_go;
  const int stride = gridDim.x * blockDim.x;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += stride) {
    // the triples were merged beforehand (pre, [3, T]) when there are few rows
    const float3 v = pre != nullptr ? make_float3(pre[t], pre[(size_t)T + t], pre[(size_t)2 * T + t])
                                    : shard_triple(part, n_groups, T, t, tgt_ws, y, v_off, Vs);
    multimem_st_f32x4(xch_mc + (size_t)rank * ld + t, make_float4(v.x, v.y, v.z, 0.f));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // this block's multicast stores before its arrival
    const unsigned prev = atomicAdd(arrivals, 1u);
    if (prev == gridDim.x - 1) {
      // every block has arrived: reset the arrival counter for the next call, then count
      // this rank once in every copy of the exchange counter
      *arrivals = 0u;
      __threadfence_system();
      multimem_red_add_release_u32(cnt_mc, 1u);
    }
    int go = 1;
    if (ld_acquire_sys_u32(cnt_local) < target) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys_u32(cnt_local) < target) {
        if (globaltimer_ns() - t0 > limit_ns) {
          record_device_error(DEV_TIMEOUT_PEER);
          go = 0;
          break;
        }
        __nanosleep(64);
      }
    }
    s_go = go;
  }
  __syncthreads();
  if (!s_go) {
    // another rank never arrived: the merged values do not exist, so this block's rows
    // get NaN instead of whatever the caller's buffers held
    for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += stride) {
      if (logp != nullptr) logp[t] = __int_as_float(0x7fc00000);
      if (norm != nullptr) {
        norm[t] = __int_as_float(0x7fc00000);
        norm[(size_t)T + t] = __int_as_float(0x7fc00000);
      }
    }
    return;
  }
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < T; t += stride) {
    float m = -INFINITY;
    for (int p = 0; p < world; ++p) m = fmaxf(m, __ldcg(&xch_local[(size_t)p * ld + t]).x);
    float s = 0.f, tgt = 0.f;
    for (int p = 0; p < world; ++p) {
      const float4 v = __ldcg(&xch_local[(size_t)p * ld + t]);
      s += v.y * expf(v.x - m);
      tgt += v.z;
    }
    if (logp != nullptr) logp[t] = tgt - m - logf(s);
    if (norm != nullptr) {
      norm[t] = m;
      norm[(size_t)T + t] = s;
    }
  }
}

// Sampler head: merge the per-unit partials of each row into the normaliser (max in
// natural units, sum exp(z - max)), the first column of the row maximum and its logp. One
// block per row (a decode batch has few rows and many partials): each thread folds a
// strided subset of the partials, then the block reduces. Ties keep the smaller column
// (the first occurrence, as argmax does).
struct HeadAcc {
  float m, s, bz;  // running max (base 2) and sum, best logit
  int bi;          // its column (-1: none yet)
};

__device__ __forceinline__ HeadAcc head_merge(HeadAcc a, HeadAcc b) {
  HeadAcc r;
  r.m = fmaxf(a.m, b.m);
  r.s = (a.m == -INFINITY ? 0.f : a.s * exp2f(a.m - r.m)) + (b.m == -INFINITY ? 0.f : b.s * exp2f(b.m - r.m));
  const bool take_b = b.bi >= 0 && (a.bi < 0 || b.bz > a.bz || (b.bz == a.bz && b.bi < a.bi));
  r.bz = take_b ? b.bz : a.bz;
  r.bi = take_b ? b.bi : a.bi;
  return r;
}

__global__ void head_finalize_kernel(const float2* __restrict__ part, const float2* __restrict__ best, int n_parts,
                                     int B, float* __restrict__ norm, int32_t* __restrict__ argmax,
                                     float* __restrict__ argmax_logp) {
  __shared__ HeadAcc warp_acc[32];
  const int t = blockIdx.x;
  HeadAcc acc{-INFINITY, 0.f, -INFINITY, -1};
  for (int g = threadIdx.x; g < n_parts; g += blockDim.x) {
    const float2 p = part[(size_t)g * B + t];
    const float2 b = best[(size_t)g * B + t];
    acc = head_merge(acc, HeadAcc{p.x, p.y, b.x, __float_as_int(b.y)});
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    HeadAcc o;
    o.m = __shfl_down_sync(0xffffffffu, acc.m, off);
    o.s = __shfl_down_sync(0xffffffffu, acc.s, off);
    o.bz = __shfl_down_sync(0xffffffffu, acc.bz, off);
    o.bi = __shfl_down_sync(0xffffffffu, acc.bi, off);
    acc = head_merge(acc, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) warp_acc[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) acc = head_merge(acc, warp_acc[w]);
    const float mx = acc.m * kLn2;
    if (norm != nullptr) {
      norm[t] = mx;
      norm[(size_t)B + t] = acc.s;
    }
    if (argmax != nullptr) argmax[t] = acc.bi;
    if (argmax_logp != nullptr) argmax_logp[t] = acc.bz - (mx + logf(acc.s));
  }
}

// logits[b, v] -= max_b + log(sum_b) in place: the full log-softmax of the sampler. Rows are
// 16-byte aligned (ld % 4 == 0, the TMA store's requirement); blockIdx.y strides the rows.
__global__ void logits_to_logprobs_kernel(float* __restrict__ logits, long long ld, int B, long long V,
                                          const float* __restrict__ norm) {
  const long long v4 = V / 4;
  for (int b = blockIdx.y; b < B; b += gridDim.y) {
    const float lse = norm[b] + logf(norm[(size_t)B + b]);
    float* row = logits + (size_t)b * ld;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < v4; i += (long long)gridDim.x * blockDim.x) {
      float4 x = reinterpret_cast<float4*>(row)[i];
      x.x -= lse;
      x.y -= lse;
      x.z -= lse;
      x.w -= lse;
      reinterpret_cast<float4*>(row)[i] = x;
    }
    for (long long v = 4 * v4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; v < V;
         v += (long long)gridDim.x * blockDim.x)
      row[v] -= lse;
  }
}

// Cross-shard combine: global max, rescaled sum, summed owned target logit.
__global__ void combine_kernel(const float* __restrict__ shard_stats, int P, int T, float* __restrict__ logp,
                               float* __restrict__ norm) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  float m = -INFINITY;
  for (int p = 0; p < P; ++p) m = fmaxf(m, shard_stats[((size_t)p * 3 + 0) * T + t]);
  float s = 0.f, tgt = 0.f;
  for (int p = 0; p < P; ++p) {
    s += shard_stats[((size_t)p * 3 + 1) * T + t] * expf(shard_stats[((size_t)p * 3 + 0) * T + t] - m);
    tgt += shard_stats[((size_t)p * 3 + 2) * T + t];
  }
  if (logp != nullptr) logp[t] = tgt - m - logf(s);
  if (norm != nullptr) {
    norm[t] = m;
    norm[(size_t)T + t] = s;
  }
}

// out[r][c] = sum_s part[s][r][c] for r < M, c < N (N % 4 == 0); bf16 or f32 output.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int S, long long M, long long N, long long Mpad,
                                     void* __restrict__ out, long long ld_out, int out_bf16) {
  const long long n4 = N / 4;
  const long long total = M * n4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  auto store = [&](long long r, long long c, const float4& acc) {
    if (out_bf16) {
      uint2 pk;
      pk.x = pack_bf16x2(acc.x, acc.y);
      pk.y = pack_bf16x2(acc.z, acc.w);
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(out) + r * ld_out + c) = pk;
    } else {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + r * ld_out + c) = acc;
    }
  };
  // Two output vectors per thread and the split loop unrolled, so several independent
  // 16-byte loads are in flight (the sum over s stays in split order).
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += 2 * stride) {
    const long long j = i + stride;
    const bool has_j = j < total;
    const long long r0 = i / n4, c0 = (i % n4) * 4;
    const long long r1 = has_j ? j / n4 : r0, c1 = has_j ? (j % n4) * 4 : c0;
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
#pragma unroll 4
    for (int s = 0; s < S; ++s) {
      const float4 v0 = *reinterpret_cast<const float4*>(part + ((size_t)s * Mpad + r0) * N + c0);
      const float4 v1 = *reinterpret_cast<const float4*>(part + ((size_t)s * Mpad + r1) * N + c1);
      a0.x += v0.x;
      a0.y += v0.y;
      a0.z += v0.z;
      a0.w += v0.w;
      a1.x += v1.x;
      a1.y += v1.y;
      a1.z += v1.z;
      a1.w += v1.w;
    }
    store(r0, c0, a0);
    if (has_j) store(r1, c1, a1);
  }
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst, long long n) {
  const long long n4 = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(src)[i];
    uint2 pk;
    pk.x = pack_bf16x2(v.x, v.y);
    pk.y = pack_bf16x2(v.z, v.w);
    reinterpret_cast<uint2*>(dst)[i] = pk;
  }
  const long long tail = n4 * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (tail < n) dst[tail] = __float2bfloat16_rn(src[tail]);
}

// ----------------------------------------------------------------------------- compaction
constexpr int kCompactBlock = 1024;  // slots per block (256 threads x 4)

__global__ void compact_count_kernel(const uint8_t* __restrict__ mask, long long slots, int* __restrict__ block_counts) {
  __shared__ int warp_sums[8];
  const long long base = (long long)blockIdx.x * kCompactBlock;
  int c = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const long long s = base + k * 256 + threadIdx.x;
    c += (s < slots && mask[s] != 0) ? 1 : 0;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < 8; ++w) t += warp_sums[w];
    block_counts[blockIdx.x] = t;
  }
}

// Exclusive scan of the per-block counts by a single 1024-thread block (warp shuffles).
__global__ void compact_scan_kernel(const int* __restrict__ block_counts, int nblocks, int* __restrict__ block_offsets,
                                    int* __restrict__ count) {
  __shared__ int warp_tot[32];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int base = 0; base < nblocks; base += 1024) {
    const int i = base + threadIdx.x;
    const int v = i < nblocks ? block_counts[i] : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += n;
    }
    if (lane == 31) warp_tot[w] = x;
    __syncthreads();
    if (w == 0) {
      int t = warp_tot[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += n;
      }
      warp_tot[lane] = t;  // inclusive
    }
    __syncthreads();
    const int warp_off = (w > 0 ? warp_tot[w - 1] : 0);
    if (i < nblocks) block_offsets[i] = carry + warp_off + x - v;
    __syncthreads();
    if (threadIdx.x == 0) carry += warp_tot[31];
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = carry;
}

// Writes idx (compact -> slot) and pos (slot -> compact or -1), preserving slot order.
__global__ void compact_write_kernel(const uint8_t* __restrict__ mask, long long slots,
                                     const int* __restrict__ block_offsets, int32_t* __restrict__ idx,
                                     int32_t* __restrict__ pos) {
  __shared__ int warp_cnt[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const long long base = (long long)blockIdx.x * kCompactBlock;
  // 256 threads, 4 passes of 256 consecutive slots; running offset across passes
  int running = block_offsets[blockIdx.x];
  for (int k = 0; k < 4; ++k) {
    const long long s = base + k * 256 + threadIdx.x;
    const bool valid = s < slots && mask[s] != 0;
    const unsigned ballot = __ballot_sync(0xffffffffu, valid);
    if (lane == 0) warp_cnt[w] = __popc(ballot);
    __syncthreads();
    int before = 0;
    for (int j = 0; j < w; ++j) before += warp_cnt[j];
    int total = before;
    for (int j = w; j < 8; ++j) total += warp_cnt[j];
    const int my = running + before + __popc(ballot & ((1u << lane) - 1u));
    if (s < slots) {
      pos[s] = valid ? my : -1;
      if (valid) idx[my] = (int32_t)s;
    }
    running += total;
    __syncthreads();
  }
}

// One warp per compact row: H_out[i] = hidden row of slot idx[i], y_out[i] = ids[slot].
__global__ void compact_gather_kernel(const int32_t* __restrict__ idx, const int* __restrict__ count, long long N,
                                      const __nv_bfloat16* __restrict__ hidden, long long bstride, long long rstride,
                                      long long row_offset, long long d, const int32_t* __restrict__ ids,
                                      __nv_bfloat16* __restrict__ H_out, int32_t* __restrict__ y_out) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const int n = *count;
  const long long vec = d / 8;  // 16-byte vectors per row (d % 8 == 0)
  for (long long i = warp_id; i < n; i += nwarps) {
    const long long slot = idx[i];
    const long long b = slot / N, j = slot % N;
    const uint4* src = reinterpret_cast<const uint4*>(hidden + b * bstride + (j + row_offset) * rstride);
    uint4* dst = reinterpret_cast<uint4*>(H_out + i * d);
    for (long long v = lane; v < vec; v += 32) dst[v] = src[v];
    if (lane == 0 && y_out != nullptr) y_out[i] = ids[slot];
  }
}

// out[s] = pos[s] >= 0 ? src[pos[s]] : 0, one warp per slot row; 16-byte vectors.
__global__ void scatter_rows_vec_kernel(const uint8_t* __restrict__ src, long long src_stride_b,
                                        const int32_t* __restrict__ pos, long long slots, long long row_bytes,
                                        uint8_t* __restrict__ out, long long out_stride_b, long long rows_per_group,
                                        long long group_stride_b) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long vec = row_bytes / 16;
  for (long long s = warp_id; s < slots; s += nwarps) {
    const int p = pos[s];
    uint4* dst = reinterpret_cast<uint4*>(out + (s / rows_per_group) * group_stride_b + (s % rows_per_group) * out_stride_b);
    if (p >= 0) {
      const uint4* sr = reinterpret_cast<const uint4*>(src + (long long)p * src_stride_b);
      for (long long v = lane; v < vec; v += 32) dst[v] = sr[v];
    } else {
      for (long long v = lane; v < vec; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    }
  }
}

// f32 rows -> bf16 rows: one warp per slot row, 8 columns (32 B in, 16 B out) per lane step.
__global__ void scatter_rows_f32_to_bf16_kernel(const float* __restrict__ src, long long src_stride,
                                                const int32_t* __restrict__ pos, long long slots, long long width,
                                                __nv_bfloat16* __restrict__ out, long long out_stride,
                                                long long rows_per_group, long long group_stride) {
  const int lane = threadIdx.x & 31;
  const long long warp_id = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const long long vec = width / 8;
  for (long long s = warp_id; s < slots; s += nwarps) {
    const int p = pos[s];
    uint4* dst = reinterpret_cast<uint4*>(out + (s / rows_per_group) * group_stride + (s % rows_per_group) * out_stride);
    if (p >= 0) {
      const float4* sr = reinterpret_cast<const float4*>(src + (long long)p * src_stride);
      for (long long v = lane; v < vec; v += 32) {
        const float4 a = sr[2 * v], b = sr[2 * v + 1];
        dst[v] = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y), pack_bf16x2(b.z, b.w));
      }
    } else {
      for (long long v = lane; v < vec; v += 32) dst[v] = make_uint4(0, 0, 0, 0);
    }
  }
}

// Barrier of `world` ranks through their signal pads (peer-mapped, zero-initialised u32
// slots; pads[p] is this process's address of rank p's pad). Rank r sets slot
// [channel][r] of every pad from 0 to 1 (waiting until the previous signal there was
// consumed), then waits for slot [channel][p] of its own pad to hold 1 and resets it, for
// every p. Waits are bounded by limit_ns; on expiry the kernel records DEV_TIMEOUT_PEER and
// returns. The system-scope fences order this rank's earlier writes (multicast reductions
// included) before its signals, and the peers' writes before what follows the barrier.
__global__ void peer_barrier_kernel(const unsigned long long* __restrict__ pads, int rank, int world, int channel,
                                    unsigned long long limit_ns) {
  const int p = threadIdx.x;
  if (p < world) {
    unsigned int* peer = reinterpret_cast<unsigned int*>(pads[p]) + (size_t)channel * world + rank;
    unsigned int* own = reinterpret_cast<unsigned int*>(pads[rank]) + (size_t)channel * world + p;
    fence_sys();
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    while (atomicCAS_system(peer, 0u, 1u) != 0u) {
      if (globaltimer_ns() - t0 > limit_ns) {
        record_device_error(DEV_TIMEOUT_PEER);
        ok = false;
        break;
      }
    }
    while (ok && atomicCAS_system(own, 1u, 0u) != 1u) {
      if (globaltimer_ns() - t0 > limit_ns) {
        record_device_error(DEV_TIMEOUT_PEER);
        break;
      }
    }
    fence_sys();
  }
  __syncthreads();
}

// Element-wise fallback layout for rows that are not 16-byte multiples (e.g. logps).
__global__ void scatter_rows_elem_kernel(const uint8_t* __restrict__ src, long long src_stride,
                                         const int32_t* __restrict__ pos, long long slots, long long width,
                                         int elem_bytes, uint8_t* __restrict__ out, long long out_stride,
                                         long long rows_per_group, long long group_stride) {
  const long long total = slots * width;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long s = i / width, c = i % width;
    const int p = pos[s];
    const long long o = (s / rows_per_group) * group_stride + (s % rows_per_group) * out_stride + c;
    if (elem_bytes == 4) {
      const float v = p >= 0 ? reinterpret_cast<const float*>(src)[(long long)p * src_stride + c] : 0.f;
      reinterpret_cast<float*>(out)[o] = v;
    } else {
      const uint16_t v = p >= 0 ? reinterpret_cast<const uint16_t*>(src)[(long long)p * src_stride + c] : (uint16_t)0;
      reinterpret_cast<uint16_t*>(out)[o] = v;
    }
  }
}

}  // namespace lpk
