// Row-staged kernel: one warp owns whole rows, for [residual-free] RMSNorm
// -> [1x128 group FP8 | per-token FP8 | no quantization] over batches with
// many rows of up to 8192 columns.
//
// Same per-element arithmetic as the pipelined kernel (pipe_kernel.cuh) and
// its interleaved layout inside each 128-vector (2 KB) block of a row: lane
// i of octet o holds vectors o*32 + i + 8k, k = 0..3, so an octet covers two
// whole 1x128 groups of the block. What changes is the unit of work. The
// pipelined kernel spreads a row over a CTA (32 elements a thread), so every
// row pays for an exchange between warps: partial sums through a ring, a
// finisher warp, inv_rms through a second ring, and a counter for releasing
// the stage. Here a warp processes its rows alone:
//
//  * each warp has one shared-memory slot; its lane 0 streams the warp's
//    next row into it with one cp.async.bulk (one mbarrier a slot);
//  * the warp pulls the whole row from the slot into registers (NB blocks of
//    4 vectors a lane: 16 NB registers, 112 at H = 7168) and, once its sum
//    of squares has used every value, refills the slot with its next row,
//    which then has nearly a whole row's processing time to land;
//  * from registers: the sum of squares (warp butterfly; every lane forms
//    inv_rms itself), then per block normalise, two 1x128 group maxima an
//    octet (three butterfly steps, two groups a step), scales, reciprocals
//    and codes; per-token scaling normalises the whole row in place, takes
//    the row maximum, then writes the codes — no second read of the row.
//
// The weights are staged once per CTA in shared memory (read by every warp
// from there: the slots leave little room for the L1 cache). No barrier and
// no shared state between the warps after the set-up, so no warp ever waits
// for another; the per-row scalar work (wait, inv_rms, pointer updates) is
// spread over H / 32 elements a lane instead of 32. A CTA is one per SM with
// up to 12 (NB > 4) or 16 warps.
//
// Waits are bounded (FusedArgs::wait_limit); a wait that gives up records
// code 1 in the device error word, and the warp lets its copy in flight land
// (bounded) before it stops. A slot is refilled only after every lane has
// read it, and only when the wait for it succeeded.
#pragma once

#include "pipe_kernel.cuh"

namespace cutie {

constexpr int kRowstageMaxNB = 8;  // 2 KB blocks a row: H <= 8192
constexpr uint32_t kRowstageBlockBytes = 2048;  // 128 vectors of 16 bytes

// Warps a CTA may hold (registers: NB blocks keep 16 NB registers a lane for
// the row).
__host__ __device__ constexpr int rowstage_max_warps(int NB) { return NB <= 4 ? 16 : 12; }

// Bytes of one row slot: whole 2 KB blocks (the tail of a partial last
// block is zeroed once and never written by the copies).
__host__ __device__ inline uint32_t rowstage_row_pad(int V) {
  return (uint32_t)((V + 127) / 128) * kRowstageBlockBytes;
}

// QM: kQGroup (1x128 groups), kQToken (one scale a row) or kQNone. NB: 2 KB
// blocks a row (V <= 128 NB; only the last block may be partial). SK: scale
// destination (pipe_kernel.cuh). Dynamic shared memory: the weights, then one
// slot a warp, each rowstage_row_pad(V) bytes.
template <int QM, int NB, int SK>
__global__ void __launch_bounds__(rowstage_max_warps(NB) * 32, 1)
    rowstage_rmsnorm_fp8_kernel(const FusedArgs a) {
  static_assert(QM == kQGroup || QM == kQToken || QM == kQNone, "mode");
  static_assert(NB >= 1 && NB <= kRowstageMaxNB, "blocks a row");
  constexpr bool kPow2 = SK != kSkF32;
  constexpr int kEsz = (SK == kSkE8 || SK == kSkE8Swz) ? 1 : 4;
  constexpr int kMaxW = rowstage_max_warps(NB);
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full_bar[kMaxW];
  __shared__ __align__(8) uint64_t w_bar;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
  const int V = a.V;
  const uint32_t row_bytes = (uint32_t)V * 16u;
  constexpr uint32_t row_pad = (uint32_t)NB * kRowstageBlockBytes;
  const uint32_t wslot = smem_addr(smem);
  const uint32_t slot = wslot + row_pad * (uint32_t)(1 + warp);
  const uint32_t bar = smem_addr(&full_bar[warp]);
  const int64_t nwarp = (int64_t)gridDim.x * W;
  const int64_t wid = (int64_t)blockIdx.x * W + warp;
  const int64_t nrows = wid < a.M ? (a.M - 1 - wid) / nwarp + 1 : 0;
  const bool full = V == NB * 128;  // no partial last block

  // the barrier array holds kMaxW warps; the host plans within it (anything
  // else is refused before any set-up)
  if (W > kMaxW || V > NB * 128 || V <= (NB - 1) * 128) {
    if (threadIdx.x == 0) atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBadLaunch);
    return;
  }

  auto issue = [&](int64_t row) {
    mbar_arrive_expect_tx(bar, row_bytes);
    bulk_g2s(slot, a.x + row * a.ldx, row_bytes, bar);
  };

  // zero the tails past the row (weights and this warp's slot): the copies
  // never write them, and every lane reads whole blocks
  if (!full) {
    for (uint32_t b = row_bytes + 4u * (uint32_t)lane; b < row_pad; b += 128u)
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(slot + b), "r"(0u) : "memory");
    if (warp == 0)
      for (uint32_t b = row_bytes + 4u * (uint32_t)lane; b < row_pad; b += 128u)
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(wslot + b), "r"(0u) : "memory");
  }
  if (lane == 0) {
    mbar_init(bar, 1);
    if (warp == 0) mbar_init(smem_addr(&w_bar), 1);
    mbar_init_fence();
  }
  __syncthreads();
  griddep_wait();  // inputs of the previous kernel are complete from here on
  griddep_launch_dependents();
  if (lane == 0) {
    if (warp == 0) {
      mbar_arrive_expect_tx(smem_addr(&w_bar), row_bytes);
      bulk_g2s(wslot, a.w, row_bytes, smem_addr(&w_bar));
    }
    if (nrows > 0) issue(wid);
  }
  const bool w_ok = __all_sync(0xffffffffu,
                               mbar_wait_bounded(smem_addr(&w_bar), 0u, a.wait_limit));

  // this lane's vector within a 2 KB block, and its 1x128 group there
  const int tvec = (lane >> 3) * 32 + (lane & 7);
  const uint32_t toff = (uint32_t)tvec * 16u;
  const int gsub = (lane >> 3) * 2 + (lane & 1);  // group within the block (8 a block)
  const bool gput = (lane & 6) == 0;              // lanes 0 and 1 of an octet
  const bool store_no = a.norm_out != nullptr;
  // vector k2 of block b lies inside the row (only the last block can fail)
  auto in_row = [&](int b, int k2) { return full || b < NB - 1 || (b * 128 + tvec + 8 * k2) < V; };

  uint32_t par = 0;
  int64_t row = wid;
  for (int64_t k = 0; k < nrows; ++k, row += nwarp) {
    const bool ok = w_ok && __all_sync(0xffffffffu, mbar_wait_bounded(bar, par, a.wait_limit));
    if (!ok) {
      // A copy never landed in time: record it, let this warp's copies in
      // flight land (bounded), and stop.
      if (lane == 0) {
        atomicCAS(&g_cutie_device_error, kDevErrNone, kDevErrBulkWaitTimeout);
        mbar_wait_bounded(bar, par, kDrainLimitCycles);
        if (warp == 0) mbar_wait_bounded(smem_addr(&w_bar), 0u, kDrainLimitCycles);
      }
      return;
    }
    // the whole row into registers
    uint32_t v[NB][4][4];
#pragma unroll
    for (int b = 0; b < NB; ++b)
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) {
        const uint4 u = ld_smem(slot + toff + (uint32_t)b * kRowstageBlockBytes + 128u * k2);
        v[b][k2][0] = u.x;
        v[b][k2][1] = u.y;
        v[b][k2][2] = u.z;
        v[b][k2][3] = u.w;
      }
    par ^= 1u;

    // sum of squares: per vector slot across the blocks, then the slots,
    // then the pair, then the butterfly
    float2 acc[4];
#pragma unroll
    for (int k2 = 0; k2 < 4; ++k2) {
      acc[k2] = sq_first(v[0][k2][0]);
#pragma unroll
      for (int j = 1; j < 4; ++j) sq_acc(acc[k2], v[0][k2][j]);
#pragma unroll
      for (int b = 1; b < NB; ++b)
#pragma unroll
        for (int j = 0; j < 4; ++j) sq_acc(acc[k2], v[b][k2][j]);
    }
#pragma unroll
    for (int k2 = 1; k2 < 4; ++k2) acc[0] = __fadd2_rn(acc[0], acc[k2]);
    // Every value read from the slot has been used by now, so the slot takes
    // the warp's next row (the proxy fence orders the lanes' reads, joined by
    // __syncwarp, before the copy engine's writes); it lands while this row
    // is processed.
    __syncwarp();
    if (lane == 0 && k + 1 < nrows) {
      fence_proxy_async_smem();
      issue(row + nwarp);
    }
    const float ss = warp_reduce<false>(__fadd_rn(acc[0].x, acc[0].y));
    // torch.rsqrt on the CPU is RN(1 / RN(sqrt(v))); the mean is RN(ss / H)
    float mean = div_rn(ss, (float)a.H, a.rcp_H);
    if (mean < 0x1p-100f) mean = __fdiv_rn(ss, (float)a.H);
    const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(mean, a.eps)));
    const float2 inv2 = make_float2(inv, inv);

    uint8_t* qrow = a.q + row * a.ldq;
    char* srow = static_cast<char*>(a.scale) + row * a.s_row * kEsz;
    uint8_t* norow = reinterpret_cast<uint8_t*>(a.norm_out) + row * a.ldn * 2;

    // block b normalised in place: bf16(bf16(r * inv) * w), the weights
    // from the CTA's shared copy (same bits as every other kernel)
    auto normalize = [&](int b) {
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) {
        const uint4 wv = ld_smem(wslot + toff + (uint32_t)b * kRowstageBlockBytes + 128u * k2);
        const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[b][k2][j] = mul_bf2(f2_to_bf2(__fmul2_rn(bf2_to_f2(v[b][k2][j]), inv2)), w4[j]);
      }
      if (store_no) {
#pragma unroll
        for (int k2 = 0; k2 < 4; ++k2)
          st_stream_if(in_row(b, k2), norow + (int64_t)(b * 128 + tvec + 8 * k2) * 16, v[b][k2]);
      }
    };
    // codes of block b (slots 0-1 with scale A, 2-3 with scale B)
    auto store_codes = [&](int b, float sa, float ra, float sb, float rb) {
      uint32_t* qthr = reinterpret_cast<uint32_t*>(qrow + (int64_t)(b * 128 + tvec) * 8);
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) {
        const float rcs = k2 < 2 ? ra : rb, ns = k2 < 2 ? -sa : -sb;
        const float2 rc2 = make_float2(rcs, rcs), nb = make_float2(ns, ns);
        float2 y[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if constexpr (kPow2)
            y[j] = __fmul2_rn(bf2_to_f2(v[b][k2][j]), rc2);  // n * 2^-e is exact
          else
            y[j] = div2_rn(bf2_to_f2(v[b][k2][j]), nb, rc2);
        }
        // 8 codes of vector tvec + 8 k2: an octet writes 64 contiguous bytes
        st_stream2_if(in_row(b, k2), qthr + 16 * k2, f4_to_e4m3x4(y[0], y[1]),
                      f4_to_e4m3x4(y[2], y[3]));
      }
    };

    if constexpr (QM == kQGroup) {
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        normalize(b);
        const uint32_t pa = absmax_bf2(vec_absmax(v[b][0]), vec_absmax(v[b][1]));
        const uint32_t pb = absmax_bf2(vec_absmax(v[b][2]), vec_absmax(v[b][3]));
        uint32_t p =
            absmax_bf2(__byte_perm(pa, pb, 0x5410), __byte_perm(pa, pb, 0x7632)) & 0x7fff7fffu;
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) p = max_bf2(p, __shfl_xor_sync(0xffffffffu, p, o));
        const float2 am = bf2_to_f2(p);
        const float sa = make_scale(am.x, kPow2), sb = make_scale(am.y, kPow2);
        float ra, rb;
        if constexpr (kPow2) {  // exact reciprocals of powers of two: negate the exponent
          ra = __uint_as_float((254u << 23) - __float_as_uint(sa));
          rb = __uint_as_float((254u << 23) - __float_as_uint(sb));
        } else {
          ra = rcp_scale(sa);
          rb = rcp_scale(sb);
        }
        const int g = b * 8 + gsub;
        const int64_t goff = ((int64_t)(g >> 2) * a.s_grp4 + (int64_t)(g & 3) * a.s_grp) * kEsz;
        put_group_scale<SK>(gput && (full || g * 16 < V), a, row, srow, goff, g,
                            (lane & 1) ? sb : sa);
        store_codes(b, sa, ra, sb, rb);
      }
      if constexpr (SK == kSkE8Swz)
        if (a.n_groups_pad > a.n_groups) zero_scale_padding(a, row, a.n_groups, lane, 32);
    } else if constexpr (QM == kQToken) {
      // normalise the whole row in place, then its maximum, then the codes
      uint32_t pm = 0u;
#pragma unroll
      for (int b = 0; b < NB; ++b) {
        normalize(b);
        pm = absmax_bf2(pm, absmax_bf2(absmax_bf2(vec_absmax(v[b][0]), vec_absmax(v[b][1])),
                                       absmax_bf2(vec_absmax(v[b][2]), vec_absmax(v[b][3]))));
      }
      pm &= 0x7fff7fffu;
      pm = max_bf2(pm, pm >> 16);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) pm = max_bf2(pm, __shfl_xor_sync(0xffffffffu, pm, o));
      const float sc = make_scale(__uint_as_float(pm << 16), kPow2);
      const float rc = kPow2 ? __uint_as_float((254u << 23) - __float_as_uint(sc)) : rcp_scale(sc);
      put_group_scale<SK>(lane == 0, a, row, srow, 0, 0, sc);
#pragma unroll
      for (int b = 0; b < NB; ++b) store_codes(b, sc, rc, sc, rc);
    } else {
#pragma unroll
      for (int b = 0; b < NB; ++b) normalize(b);
    }
  }
  if constexpr (SK == kSkE8Swz)  // swizzled-layout padding rows: scales only
    for (int64_t r = wid + nrows * nwarp; r < a.M_pad; r += nwarp) zero_scale_padding(a, r, 0, lane, 32);
  // a warp with no rows still waited for the weights; nothing is in flight
}

}  // namespace cutie
