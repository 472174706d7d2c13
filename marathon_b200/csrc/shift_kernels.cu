// shift_kernels.cu — sm_100a kernels of the position-shifted KV reuse path.
//
// Load (store -> paged cache, K re-rotated by each run's delta) and save
// (paged cache -> store, bit copy) are one templated persistent kernel.  A
// launch covers every (layer, run, token tile) of a batch: multi-layer,
// multi-run and multi-session work is a single launch.
//
// Work decomposition.  A tile is up to `tile_tokens` consecutive tokens of
// one run in one layer.  Tiles are numbered layer-major
// (w = layer * tiles_per_layer + tile) and CTAs stride over them, so
// neighbouring CTAs read neighbouring store rows and write neighbouring
// paged blocks.  The run owning a tile is found by a uniform binary search
// over the runs' tile_begin prefix.
//
// Per tile the CTA first resolves every token's paged offset (slot -> block,
// offset; bounds-checked, bad tokens flagged and skipped) into shared memory
// and stages the run's cos/sin table there.  Then G = head_size/(2*VEC)
// threads cooperate on one (token, head) unit: each thread moves two 16-byte
// K vectors and two 16-byte V vectors.  For K the two vectors are RoPE
// partners (elements i and i + rotary/2), so the rotation
//     out[i]        = k[i] * cos[i] - k[i+half] * sin[i]
//     out[i + half] = k[i+half] * cos[i] + k[i] * sin[i]
// needs no shuffle.  Every HBM access is a 128-bit coalesced load or store
// and every byte is read once and written once.
//
// Arithmetic follows the reference's torch path term by term
// (src/marathon/shift_kernels.py:153-156): two fp32 products, rounded
// separately, then one fp32 add; no FMA contraction (__fmul_rn/__fadd_rn), so
// the fp32 value before the final rounding is bit-identical to the CPU
// computation and the stored element is its round-to-nearest-even.  E4M3:
// the layer's K scale cancels between dequantisation and requantisation, so
// the codes' values are rotated (fp32, fused multiply-add) and rounded once to
// e4m3 (saturating at +-448, RNE): within one e4m3 step of the step-by-step
// dequantise -> rotate -> divide result.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/marathon_shift.h"

// Tuning knobs (compile-time; the defaults are the measured best on B200):
//   MSHIFT_MIN_BLOCKS  resident CTAs per SM requested from ptxas (register cap)
//   MSHIFT_UNITS       (token, head) units each thread keeps in flight
//   MSHIFT_LOAD_HINT   0: ld.global.cs  1: ld.global.nc  2: ld.global.nc.L1::no_allocate.L2::256B
//   MSHIFT_STORE_HINT  0: st.global.cs  1: st.global (write-back)
#ifndef MSHIFT_MIN_BLOCKS
#define MSHIFT_MIN_BLOCKS 1
#endif
#ifndef MSHIFT_UNITS
#define MSHIFT_UNITS 2
#endif
#ifndef MSHIFT_LOAD_HINT
#define MSHIFT_LOAD_HINT 0
#endif
#ifndef MSHIFT_STORE_HINT
#define MSHIFT_STORE_HINT 0
#endif

namespace mshift {

constexpr int kThreads = 256;  // threads per CTA
constexpr int kMaxTile = 512;  // tokens per tile, upper bound (smem sizing)
constexpr int kMaxDevices = 64;

struct alignas(16) Vec {
  uint32_t w[4];
};

__device__ __forceinline__ Vec load_vec(const void* p) {
#if MSHIFT_LOAD_HINT == 0
  const uint4 r = __ldcs(reinterpret_cast<const uint4*>(p));
  return Vec{{r.x, r.y, r.z, r.w}};
#elif MSHIFT_LOAD_HINT == 1
  const uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
  return Vec{{r.x, r.y, r.z, r.w}};
#else
  Vec v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
      : "l"(p));
  return v;
#endif
}

__device__ __forceinline__ void store_vec(void* p, const Vec& v) {
#if MSHIFT_STORE_HINT == 0
  __stcs(reinterpret_cast<uint4*>(p), make_uint4(v.w[0], v.w[1], v.w[2], v.w[3]));
#else
  *reinterpret_cast<uint4*>(p) = make_uint4(v.w[0], v.w[1], v.w[2], v.w[3]);
#endif
}

// ---------------------------------------------------------------- element types
// Each type converts one 32-bit word of a 16-byte vector (kPer elements) to
// fp32 and back, rounding to nearest even.
struct Bf16 {
  static constexpr int kBytes = 2, kVec = 8, kPer = 2;
  static constexpr bool kScaled = false;
  __device__ static void unpack(uint32_t w, float* f) {
    f[0] = __uint_as_float(w << 16);
    f[1] = __uint_as_float(w & 0xffff0000u);
  }
  __device__ static uint32_t pack(const float* f) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f[0], f[1]);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};

struct F16 {
  static constexpr int kBytes = 2, kVec = 8, kPer = 2;
  static constexpr bool kScaled = false;
  __device__ static void unpack(uint32_t w, float* f) {
    const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w));
    f[0] = p.x;
    f[1] = p.y;
  }
  __device__ static uint32_t pack(const float* f) {
    const __half2 h = __floats2half2_rn(f[0], f[1]);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
};

struct F32 {
  static constexpr int kBytes = 4, kVec = 4, kPer = 1;
  static constexpr bool kScaled = false;
  __device__ static void unpack(uint32_t w, float* f) { f[0] = __uint_as_float(w); }
  __device__ static uint32_t pack(const float* f) { return __float_as_uint(f[0]); }
};

struct E4m3 {
  static constexpr int kBytes = 1, kVec = 16, kPer = 4;
  static constexpr bool kScaled = true;
  __device__ static void unpack(uint32_t w, float* f) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const __nv_fp8x2_storage_t pair = static_cast<__nv_fp8x2_storage_t>((w >> (16 * j)) & 0xffffu);
      const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
      const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&hr));
      f[2 * j] = p.x;
      f[2 * j + 1] = p.y;
    }
  }
  __device__ static uint32_t pack(const float* f) {
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(f[0], f[1]), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(f[2], f[3]), __NV_SATFINITE, __NV_E4M3);
    return (lo & 0xffffu) | ((hi & 0xffffu) << 16);
  }
};

// e4m3: dequantise with the layer's K scale s, rotate, requantise with the
// same s.  The scale cancels: (code*s*c - code'*s*sn) / s = code*c - code'*sn,
// so the kernel rotates the codes' values directly and rounds once to e4m3
// (saturating at +-448, nearest even).  In fp32 the result differs from the
// dequantise -> rotate -> divide sequence by a few fp32 ulps of the terms
// (|terms| <= 448), far below half the smallest e4m3 step (2^-10), so the two
// codes agree except next to an e4m3 rounding boundary, where they are one
// step apart: the north star's tolerance for FP8 (1 e4m3 step).
__device__ __forceinline__ uint32_t cvt_e4m3x2(float2 v) {
  return static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(v, __NV_SATFINITE, __NV_E4M3));
}

// Rotate one 32-bit word pair of e4m3 codes (elements 4w..4w+3 of each half):
// ra = x*c - y*sn and rb = y*c + x*sn, as packed fp32x2 products and fused
// multiply-adds.
__device__ __forceinline__ void rotate_word_e4m3(uint32_t& aw, uint32_t& bw, const float* cs,
                                                 const float* sn) {
  float x[4], y[4];
  E4m3::unpack(aw, x);
  E4m3::unpack(bw, y);
  const float4 c4 = *reinterpret_cast<const float4*>(cs);
  const float4 s4 = *reinterpret_cast<const float4*>(sn);
  const float2 c01 = make_float2(c4.x, c4.y), c23 = make_float2(c4.z, c4.w);
  const float2 s01 = make_float2(s4.x, s4.y), s23 = make_float2(s4.z, s4.w);
  const float2 x01 = make_float2(x[0], x[1]), x23 = make_float2(x[2], x[3]);
  const float2 y01 = make_float2(y[0], y[1]), y23 = make_float2(y[2], y[3]);
  const float2 ys01 = __fmul2_rn(y01, s01), ys23 = __fmul2_rn(y23, s23);
  const float2 xs01 = __fmul2_rn(x01, s01), xs23 = __fmul2_rn(x23, s23);
  const float2 ra01 = __ffma2_rn(x01, c01, make_float2(-ys01.x, -ys01.y));
  const float2 ra23 = __ffma2_rn(x23, c23, make_float2(-ys23.x, -ys23.y));
  const float2 rb01 = __ffma2_rn(y01, c01, xs01);
  const float2 rb23 = __ffma2_rn(y23, c23, xs23);
  aw = cvt_e4m3x2(ra01) | (cvt_e4m3x2(ra23) << 16);
  bw = cvt_e4m3x2(rb01) | (cvt_e4m3x2(rb23) << 16);
}

// Rotate one pair of partner vectors in place: `a` holds elements
// [i0, i0+VEC) of the first rotary half, `b` the same elements of the second.
// Works one 32-bit word (kPer elements) at a time to keep few values live.
// 16/32-bit types: the products of two elements share one packed fp32x2
// multiply (each lane rounds on its own), the sums are scalar, so the results
// are those of the scalar __fmul_rn / __fsub_rn / __fadd_rn sequence -- the
// reference's operation order, rounded once to the cache type.
template <class E>
__device__ __forceinline__ void rotate_pair(Vec& a, Vec& b, const float* cs, const float* sn) {
  if constexpr (E::kScaled) {
#pragma unroll
    for (int w = 0; w < 4; ++w) rotate_word_e4m3(a.w[w], b.w[w], cs + 4 * w, sn + 4 * w);
  } else {
    constexpr int P = E::kPer;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      float x[P], y[P];
      E::unpack(a.w[w], x);
      E::unpack(b.w[w], y);
      if constexpr (P == 1) {
        const float c = cs[w], s = sn[w];
        const float xe = x[0], ye = y[0];
        x[0] = __fsub_rn(__fmul_rn(xe, c), __fmul_rn(ye, s));
        y[0] = __fadd_rn(__fmul_rn(ye, c), __fmul_rn(xe, s));
      } else {
#pragma unroll
        for (int j = 0; j < P / 2; ++j) {
          const float2 c = *reinterpret_cast<const float2*>(cs + P * w + 2 * j);
          const float2 s = *reinterpret_cast<const float2*>(sn + P * w + 2 * j);
          const float2 x2 = make_float2(x[2 * j], x[2 * j + 1]);
          const float2 y2 = make_float2(y[2 * j], y[2 * j + 1]);
          // packed products, scalar adds: __fadd_rn / __fsub_rn are never merged
          // with a multiply, so every product is rounded before it is added
          const float2 xc = __fmul2_rn(x2, c), ys = __fmul2_rn(y2, s);
          const float2 yc = __fmul2_rn(y2, c), xs = __fmul2_rn(x2, s);
          const float2 ra = make_float2(__fsub_rn(xc.x, ys.x), __fsub_rn(xc.y, ys.y));
          const float2 rb = make_float2(__fadd_rn(yc.x, xs.x), __fadd_rn(yc.y, xs.y));
          x[2 * j] = ra.x, x[2 * j + 1] = ra.y;
          y[2 * j] = rb.x, y[2 * j + 1] = rb.y;
        }
      }
      a.w[w] = E::pack(x);
      b.w[w] = E::pack(y);
    }
  }
}

// ------------------------------------------------------------------ arguments
struct KArgs {
  const mshift_run* runs;  // device; nullptr selects the single-run fields below
  int32_t n_runs;
  int32_t tile_tokens;
  int32_t tiles_per_layer;
  int32_t n_layers;
  void* const* store_ptrs;   // [n_sessions * n_layers]
  const int64_t* store_caps; // [n_sessions]
  int32_t n_sessions;
  int32_t block_size;
  int64_t st_tok, st_head;   // store strides (elements)
  void* const* k_ptrs;       // [n_layers]
  void* const* v_ptrs;
  int64_t blk_stride, off_stride, head_stride, num_slots;
  int32_t heads;
  int32_t n_tables;
  const float* tables;       // [n_tables][2][half]
  uint32_t* err;
  // diagnostic hook of the TMA load kernel: 0 = normal; n > 0 bounds every
  // consumer warp's first full-barrier wait to n - 1 rounds
  uint32_t first_wait;
  // 1: CTAs claim tiles from a counter kept in bits 8..31 of *err (see
  // claim_tile); 0: CTA b takes tiles b, b + grid, b + 2*grid, ...
  int32_t dyn;
  // single run, single layer (runs == nullptr)
  mshift_run run0;
  void* store0;
  int64_t cap0;
  void* k0;
  void* v0;
  const float* table0;
};

__device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Programmatic dependent launch.  The batched kernels are launched so that
// their CTAs may become resident while the preceding kernel in the stream
// (the rotation-table kernel) is still running; each thread first waits
// here until that kernel has completed and its writes are visible.  Launched
// without the attribute (or after a copy) the wait returns at once.
__device__ __forceinline__ void wait_prior_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Lets the dependent kernel of the stream start launching its CTAs now; it
// still reads nothing of ours before this grid has completed.
__device__ __forceinline__ void allow_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Dynamic tile scheduling.  The caller zeroes the status word *err before
// the launch; its low 8 bits collect MSHIFT_EBIT_* flags and its high 24 bits
// count claimed tiles.  Every claim adds 256 and returns the tile index; each
// CTA claims until it draws an index >= total, so exactly total + gridDim.x
// claims are made and the one that draws total + gridDim.x - 1 is the last
// claim of the launch: it clears the counter bits, leaving only the flags
// (the caller reads *err after the launch exactly as with static tiles).
// Tiles then go to whichever CTA is free first, so a launch ends within one
// tile of its fastest CTA instead of after its slowest stride.
__device__ __forceinline__ int claim_tile(uint32_t* err, int total) {
  const uint32_t old = atomicAdd(err, 256u);
  const int t = static_cast<int>(old >> 8);
  if (t == total + static_cast<int>(gridDim.x) - 1) atomicAnd(err, 0xFFu);
  return t;
}

// One templated kernel for both directions.
//   SAVE = false: store rows -> paged cache, K rotated (load)
//   SAVE = true : paged cache -> store rows, bit copy (save)
template <class E, int D, int ROT, bool SAVE>
__global__ void __launch_bounds__(kThreads, MSHIFT_MIN_BLOCKS) move_kernel(const KArgs a) {
  wait_prior_grid();
  // the next turn's table kernel may launch now: it computes its tables while
  // this launch runs and waits for this launch to complete before it ends
  allow_dependents();
  constexpr int ES = E::kBytes;
  constexpr int VEC = E::kVec;
  constexpr int NV = D / VEC;      // 16-byte vectors per K (or V) row
  constexpr int HALF = ROT / 2;
  constexpr int NP = HALF / VEC;   // rotating partner pairs per row
  constexpr int G = NV / 2;        // threads per (token, head) unit
  constexpr int UPP = kThreads / G;
  static_assert(D % (2 * VEC) == 0, "head_size must hold an even number of 16-byte vectors");
  static_assert(HALF % VEC == 0 && NP <= G, "rotary half must be whole vectors");
  static_assert(kThreads % G == 0, "threads per unit must divide the CTA");

  __shared__ int64_t s_off[kMaxTile];
  __shared__ __align__(16) float s_cs[HALF > 0 ? HALF : 4];
  __shared__ __align__(16) float s_sn[HALF > 0 ? HALF : 4];
  __shared__ int s_next;  // the tile claimed for this CTA's next iteration

  const int g = threadIdx.x % G;
  const int u_first = threadIdx.x / G;
  // vector indices this thread moves in every K row: a partner pair when
  // g < NP, else two pass-through vectors of the non-rotary tail.
  const int ka = g < NP ? g : g + NP;
  const int kb = g < NP ? g + NP : g + G;
  const int total = a.tiles_per_layer * a.n_layers;

  int w = blockIdx.x;
  if (a.dyn) {
    if (threadIdx.x == 0) s_next = claim_tile(a.err, total);
    __syncthreads();
    w = s_next;
  }
  // the next tile is claimed while this one is processed; s_next is written
  // between the tile's two barriers and read after the second, and every
  // thread has read it before the next iteration's first barrier
  int prev = -1;
  for (; w < total; w = a.dyn ? s_next : w + static_cast<int>(gridDim.x)) {
    // a CTA's claims strictly increase within a launch; one that does not
    // means the counter was reset under it (a status word shared with another
    // launch in flight): stop with an error instead of taking tiles again
    if (w <= prev) {
      if (threadIdx.x == 0) atomicOr(a.err, MSHIFT_EBIT_CLAIM);
      break;
    }
    prev = w;
    const int layer = w / a.tiles_per_layer;
    const int tile = w - layer * a.tiles_per_layer;

    mshift_run run;
    char* store;
    int64_t cap;
    char* kbase;
    char* vbase;
    const float* tab = nullptr;
    bool ok_desc = true;
    uint32_t bits = 0;
    if (a.runs != nullptr) {
      int lo = 0, hi = a.n_runs - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.runs[mid].tile_begin <= tile) lo = mid; else hi = mid - 1;
      }
      run = a.runs[lo];
      const bool sess = run.session >= 0 && run.session < a.n_sessions;
      store = sess ? static_cast<char*>(a.store_ptrs[(int64_t)run.session * a.n_layers + layer])
                   : nullptr;
      cap = sess ? a.store_caps[run.session] : 0;
      if (!sess || store == nullptr || !aligned16(store)) { ok_desc = false; bits |= MSHIFT_EBIT_SESSION; }
      kbase = static_cast<char*>(a.k_ptrs[layer]);
      vbase = static_cast<char*>(a.v_ptrs[layer]);
      if (!SAVE) {
        if (run.table >= 0 && run.table < a.n_tables) tab = a.tables + (int64_t)run.table * 2 * HALF;
        else if (run.table != -1) { ok_desc = false; bits |= MSHIFT_EBIT_TABLE; }
      }
    } else {
      run = a.run0;
      store = static_cast<char*>(a.store0);
      cap = a.cap0;
      kbase = static_cast<char*>(a.k0);
      vbase = static_cast<char*>(a.v0);
      tab = SAVE ? nullptr : a.table0;
    }
    if (kbase == nullptr || vbase == nullptr || !aligned16(kbase) || !aligned16(vbase)) {
      ok_desc = false;
      bits |= MSHIFT_EBIT_SLOT;
    }
    const int t0 = (tile - run.tile_begin) * a.tile_tokens;
    const int nt = min(a.tile_tokens, run.len - t0);
    const bool tile_ok = ok_desc && nt > 0 && t0 >= 0;

    __syncthreads();  // the previous tile is done with s_off / s_cs / s_sn / s_next
    if (threadIdx.x == 0) {
      if (bits) atomicOr(a.err, bits);
      if (a.dyn) s_next = claim_tile(a.err, total);
    }
    if (tile_ok) {
      for (int t = threadIdx.x; t < nt; t += kThreads) {
        const int64_t spos = run.store_start + t0 + t;
        int64_t slot;
        bool slot_ok = true;
        if (run.slots != nullptr) {
          slot = run.slots[t0 + t];
        } else {
          const int64_t pos = run.paged_start + t0 + t;
          const int64_t bi = pos >= 0 ? pos / a.block_size : -1;
          slot_ok = bi >= 0 && bi < run.block_table_len;
          slot = slot_ok ? (int64_t)run.block_table[bi] * a.block_size + pos % a.block_size : -1;
        }
        slot_ok = slot_ok && slot >= 0 && slot < a.num_slots;
        const bool store_ok = spos >= 0 && spos < cap;
        s_off[t] = (slot_ok && store_ok)
                       ? (slot / a.block_size) * a.blk_stride + (slot % a.block_size) * a.off_stride
                       : -1;
        if (!slot_ok || !store_ok)
          atomicOr(a.err, (slot_ok ? 0u : MSHIFT_EBIT_SLOT) | (store_ok ? 0u : MSHIFT_EBIT_STORE));
      }
      if (!SAVE && HALF > 0 && tab != nullptr) {
        for (int i = threadIdx.x; i < HALF; i += kThreads) {
          s_cs[i] = tab[i];
          s_sn[i] = tab[HALF + i];
        }
      }
    }
    __syncthreads();
    if (!tile_ok) continue;

    const bool rotate = !SAVE && HALF > 0 && tab != nullptr && g < NP;
    const int nu = nt * a.heads;
    // units in the order of the side being written, so neighbouring threads
    // store neighbouring rows: a load writes the paged cache, head-major when a
    // head's tokens are adjacent there (HND); a save writes the token-major store
    const bool head_major = !SAVE && a.head_stride > a.off_stride;
    const int64_t row0 = run.store_start + t0;
    constexpr int U = MSHIFT_UNITS;
    for (int u = u_first; u < nu; u += U * UPP) {
      // U units per iteration: all 4*U loads are issued before any store
      Vec k[U][2], v[U][2];
      char* sp[U];
      char* kp[U];
      char* vp[U];
      bool live[U];
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int uu = u + q * UPP;
        live[q] = false;
        if (uu < nu) {
          int t, h;
          if (head_major) {
            h = uu / nt;
            t = uu - h * nt;
          } else {
            t = uu / a.heads;
            h = uu - t * a.heads;
          }
          const int64_t off = s_off[t];
          if (off >= 0) {
            live[q] = true;
            sp[q] = store + ((row0 + t) * a.st_tok + (int64_t)h * a.st_head) * ES;
            kp[q] = kbase + (off + (int64_t)h * a.head_stride) * ES;
            vp[q] = vbase + (off + (int64_t)h * a.head_stride) * ES;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < U; ++q) {
        if (!live[q]) continue;
        if (SAVE) {
          k[q][0] = load_vec(kp[q] + ka * 16);
          k[q][1] = load_vec(kp[q] + kb * 16);
          v[q][0] = load_vec(vp[q] + g * 16);
          v[q][1] = load_vec(vp[q] + (g + G) * 16);
        } else {
          k[q][0] = load_vec(sp[q] + ka * 16);
          k[q][1] = load_vec(sp[q] + kb * 16);
          v[q][0] = load_vec(sp[q] + D * ES + g * 16);
          v[q][1] = load_vec(sp[q] + D * ES + (g + G) * 16);
        }
      }
#pragma unroll
      for (int q = 0; q < U; ++q) {
        if (!live[q]) continue;
        if (rotate)
          rotate_pair<E>(k[q][0], k[q][1], s_cs + g * VEC, s_sn + g * VEC);
        if (SAVE) {
          store_vec(sp[q] + ka * 16, k[q][0]);
          store_vec(sp[q] + kb * 16, k[q][1]);
          store_vec(sp[q] + D * ES + g * 16, v[q][0]);
          store_vec(sp[q] + D * ES + (g + G) * 16, v[q][1]);
        } else {
          store_vec(kp[q] + ka * 16, k[q][0]);
          store_vec(kp[q] + kb * 16, k[q][1]);
          store_vec(vp[q] + g * 16, v[q][0]);
          store_vec(vp[q] + (g + G) * 16, v[q][1]);
        }
      }
    }
  }
}

// ----------------------------------------------------------- TMA bulk load
//
// Load direction when every store row is dense ([heads][2*head_size], rows
// back to back): a tile's store rows are one contiguous range, so they reach
// shared memory as ONE cp.async.bulk (TMA) per stage, completing on an
// mbarrier.  Each CTA keeps a ring of bulk_stages<E>() stages in flight.  A
// producer warp prepares each stage (run lookup, per-token slot offsets, the
// run's cos/sin row) and its lane 0 issues the bulk copy; eight consumer
// warps rotate K from shared memory and write K and V with 128-bit stores,
// then release the stage through its "empty" mbarrier.  A caller tile of
// `tile_tokens` tokens is split into parts that fit one stage; the producer
// claims whole tiles as move_kernel does (dynamic, one claim per tile) and
// publishes their parts in order, then an end-of-work stage that sends the
// consumers out.  Every copy is a plain per-CTA copy from this GPU's own memory.
// Per element type (measured best on B200, c2/c3 turns): three stages of
// 24 KiB, two CTAs per SM; eight consumer warps for 16/32-bit types, four for
// e4m3 (c3: 0.728 ms a turn against 0.750 with eight warps and 32 KiB stages,
// 0.743 with four stages of 16 KiB).  MSHIFT_BULK_STAGES, MSHIFT_BULK_STAGE_KB,
// MSHIFT_BULK_CONSUMER_WARPS and MSHIFT_BULK_MIN_BLOCKS override every type
// (tuning sweeps).
template <class E>
struct BulkCfg {
  static constexpr int kStages = 3;
  static constexpr int kStageBytes = 24 * 1024;
  static constexpr int kConsumerWarps = E::kScaled ? 4 : 8;
  static constexpr int kMinBlocks = E::kScaled ? 3 : 2;
};
#ifdef MSHIFT_BULK_STAGES
constexpr int kBulkStagesOverride = MSHIFT_BULK_STAGES;
#else
constexpr int kBulkStagesOverride = 0;
#endif
#ifdef MSHIFT_BULK_STAGE_KB
constexpr int kBulkStageBytesOverride = MSHIFT_BULK_STAGE_KB * 1024;
#else
constexpr int kBulkStageBytesOverride = 0;
#endif
template <class E>
__host__ __device__ constexpr int bulk_stages() {
  return kBulkStagesOverride ? kBulkStagesOverride : BulkCfg<E>::kStages;
}
template <class E>
__host__ __device__ constexpr int bulk_stage_bytes() {
  return kBulkStageBytesOverride ? kBulkStageBytesOverride : BulkCfg<E>::kStageBytes;
}
constexpr int kBulkMaxStages = 8;
constexpr int kBulkMaxPart = 128;          // tokens per stage, upper bound
constexpr uint32_t kWaitLimit = 1u << 18;  // try_wait rounds before giving up (seconds)

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One try_wait round: the thread may sleep up to kWaitHintNs for the phase to
// complete instead of spinning (fewer issue slots spent waiting).
constexpr uint32_t kWaitHintNs = 20000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(kWaitHintNs)
      : "memory");
  return done != 0;
}

// Bounded wait: false after `limit` rounds (the caller flags and drains), or
// as soon as another warp of the CTA has aborted (`abort` non-null and set).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          uint32_t limit = kWaitLimit,
                                          const volatile int* abort = nullptr) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort != nullptr && *abort) return false;
  }
  return false;
}

// The same wait taken by a whole warp: true only if every lane's wait
// succeeded, so the warp's lanes always take the same branch afterwards.
__device__ __forceinline__ bool warp_mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit,
                                               const volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, limit, abort);
  return __all_sync(0xffffffffu, ok);
}

// Whether any warp of the CTA has aborted, as one answer for the whole warp.
__device__ __forceinline__ bool warp_saw_abort(const volatile int* abort) {
  return __any_sync(0xffffffffu, *abort != 0);
}

// Named barrier 1 over the whole CTA (barrier 0 is __syncthreads); the
// non-aligned form, entered after the warp has reconverged.
__device__ __forceinline__ void cta_barrier_1(int threads) {
  __syncwarp();
  asm volatile("barrier.sync 1, %0;" ::"r"(threads) : "memory");
}

__device__ __forceinline__ void bulk_to_smem(void* dst, const void* src, uint32_t bytes,
                                             uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ Vec lds_vec(const unsigned char* p) {
  Vec v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
               : "r"(smem_addr(p)));
  return v;
}

struct BulkMeta {
  char* kbase;
  char* vbase;
  int nt;      // tokens staged (0: nothing to do for this stage)
  int rotate;  // the stage's table row is valid
};

#ifndef MSHIFT_BULK_UNITS_E4M3
#define MSHIFT_BULK_UNITS_E4M3 1
#endif
constexpr int kBulkUnitsE4m3 = MSHIFT_BULK_UNITS_E4M3;
#ifdef MSHIFT_BULK_CONSUMER_WARPS
constexpr int kBulkWarpsOverride = MSHIFT_BULK_CONSUMER_WARPS;
#else
constexpr int kBulkWarpsOverride = 0;
#endif
#ifdef MSHIFT_BULK_MIN_BLOCKS
constexpr int kBulkMinBlocksOverride = MSHIFT_BULK_MIN_BLOCKS;
#else
constexpr int kBulkMinBlocksOverride = 0;
#endif
// warps that rotate and store, the CTA (those + one producer warp), and the
// resident CTAs per SM the register allocation is sized for
template <class E>
__host__ __device__ constexpr int bulk_consumer_warps() {
  return kBulkWarpsOverride ? kBulkWarpsOverride : BulkCfg<E>::kConsumerWarps;
}
template <class E>
__host__ __device__ constexpr int bulk_threads() {
  return bulk_consumer_warps<E>() * 32 + 32;
}
template <class E>
__host__ __device__ constexpr int bulk_min_blocks() {
  return kBulkMinBlocksOverride ? kBulkMinBlocksOverride : BulkCfg<E>::kMinBlocks;
}

template <class E, int D, int ROT>
__global__ void __launch_bounds__(bulk_threads<E>(), bulk_min_blocks<E>()) bulk_load_kernel(
    const KArgs a, int parts, int part_tokens) {
  wait_prior_grid();
  allow_dependents();  // as in move_kernel: the next turn's table kernel may launch
  constexpr int kBulkConsumerWarps = bulk_consumer_warps<E>();
  constexpr int kBulkConsumers = kBulkConsumerWarps * 32;
  constexpr int kBulkThreads = bulk_threads<E>();
  constexpr int ES = E::kBytes;
  constexpr int VEC = E::kVec;
  constexpr int NV = D / VEC;
  constexpr int HALF = ROT / 2;
  constexpr int NP = HALF / VEC;
  constexpr int G = NV / 2;
  constexpr int UPP = kBulkConsumers / G;
  constexpr int NS = bulk_stages<E>();
  static_assert(NS >= 2 && NS <= kBulkMaxStages, "stage ring of 2..8");
  constexpr int TH = HALF > 0 ? HALF : 4;

  extern __shared__ __align__(128) unsigned char s_data[];
  __shared__ __align__(8) uint64_t s_full[NS];   // producer -> consumers: stage filled
  __shared__ __align__(8) uint64_t s_empty[NS];  // consumers -> producer: stage drained
  __shared__ BulkMeta s_meta[NS];
  __shared__ int64_t s_off[NS][kBulkMaxPart];
  __shared__ __align__(16) float s_tab[NS][2 * TH];
  __shared__ volatile int s_abort;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t row_bytes = (int64_t)a.heads * 2 * D * ES;
  const int64_t stage_bytes = (int64_t)part_tokens * row_bytes;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_empty[s], kBulkConsumerWarps);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();  // the warps part ways below and meet again only at the end

  if (warp == kBulkConsumerWarps) {
    // ------------------------------------------------------------ producer
    // The run and its layer's pointers change only every few items (items
    // are layer-major), so they are looked up once and kept in registers.
    int cur_run = -1, cur_layer = -1, next_begin = 0;
    mshift_run run{};
    const char* store = nullptr;
    int64_t cap = 0;
    char* kbase = nullptr;
    char* vbase = nullptr;
    const float* tab = nullptr;
    uint32_t desc_bits = 0;
    bool desc_ok = false;
    int k = 0;  // stages published so far (the end-of-work stage included)
    // The producer takes whole tiles -- claimed (dynamic) or this CTA's stride
    // of tiles (static) -- and publishes their parts in order, so a launch
    // makes one claim per tile, not per stage.  A claim runs one tile ahead:
    // lane 0 issues the next claim as soon as it has read the current one, so
    // the atomic's round trip overlaps the tile's stages.  Same protocol as
    // claim_tile: claims stop at the first index >= tiles, and whoever draws
    // tiles + gridDim.x - 1 clears the counter bits.
    const int tiles = a.tiles_per_layer * a.n_layers;
    int w = 0;         // the current tile
    int part = parts;  // its next part (parts: take a new tile)
    int taken = 0;     // tiles this CTA has taken
    bool done = false;
    uint32_t ahead = 0;
    if (a.dyn && lane == 0) ahead = atomicAdd(a.err, 256u);
    for (;; ++k) {
      const int s = k % NS;
      if (part == parts) {
        int64_t next;
        if (a.dyn) {
          int c = 0;
          if (lane == 0) {
            c = static_cast<int>(ahead >> 8);
            if (c == tiles + static_cast<int>(gridDim.x) - 1) atomicAnd(a.err, 0xFFu);
            if (c < tiles) ahead = atomicAdd(a.err, 256u);
          }
          next = __shfl_sync(0xffffffffu, c, 0);
          // claims strictly increase within a launch (see move_kernel)
          if (next <= w && taken > 0) {
            if (lane == 0) atomicOr(a.err, MSHIFT_EBIT_CLAIM);
            next = tiles;
          }
          ++taken;
        } else {
          next = (int64_t)blockIdx.x + (int64_t)taken * gridDim.x;
          ++taken;
        }
        done = next >= tiles;
        w = done ? 0 : static_cast<int>(next);
        part = 0;
      }
      if (warp_saw_abort(&s_abort)) break;  // a consumer warp gave up: issue nothing more
      if (k >= NS) {
        if (!warp_mbar_wait(&s_empty[s], ((k / NS) - 1) & 1, kWaitLimit, &s_abort)) {
          if (lane == 0) atomicOr(a.err, MSHIFT_EBIT_TIMEOUT);
          s_abort = 1;
          break;
        }
      }
      if (done) {
        // no more tiles: an end-of-work stage (nt = -1) sends the consumers out
        if (lane == 0) {
          s_meta[s].nt = -1;
          mbar_arrive(&s_full[s]);
        }
        ++k;
        break;
      }
      const int this_part = part++;
      const int layer = w / a.tiles_per_layer;
      const int tile = w - layer * a.tiles_per_layer;
      const bool same_run = cur_run >= 0 && tile >= run.tile_begin && tile < next_begin;
      if (!same_run) {
        int lo = 0, hi = a.n_runs - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (a.runs[mid].tile_begin <= tile) lo = mid; else hi = mid - 1;
        }
        cur_run = lo;
        run = a.runs[lo];
        next_begin = lo + 1 < a.n_runs ? a.runs[lo + 1].tile_begin : a.tiles_per_layer;
      }
      if (!same_run || layer != cur_layer) {
        cur_layer = layer;
        desc_bits = 0;
        desc_ok = true;
        const bool sess = run.session >= 0 && run.session < a.n_sessions;
        store = sess ? static_cast<const char*>(
                           a.store_ptrs[(int64_t)run.session * a.n_layers + layer])
                     : nullptr;
        cap = sess ? a.store_caps[run.session] : 0;
        if (!sess || store == nullptr || !aligned16(store)) {
          desc_ok = false;
          desc_bits |= MSHIFT_EBIT_SESSION;
        }
        kbase = static_cast<char*>(a.k_ptrs[layer]);
        vbase = static_cast<char*>(a.v_ptrs[layer]);
        if (kbase == nullptr || vbase == nullptr || !aligned16(kbase) || !aligned16(vbase)) {
          desc_ok = false;
          desc_bits |= MSHIFT_EBIT_SLOT;
        }
        tab = nullptr;
        if (run.table >= 0 && run.table < a.n_tables) tab = a.tables + (int64_t)run.table * 2 * HALF;
        else if (run.table != -1) { desc_ok = false; desc_bits |= MSHIFT_EBIT_TABLE; }
      }
      uint32_t bits = desc_bits;
      const bool ok = desc_ok;
      const int t_tile = (tile - run.tile_begin) * a.tile_tokens;
      const int t0 = t_tile + this_part * part_tokens;
      const int nt = min(min(part_tokens, a.tile_tokens - this_part * part_tokens), run.len - t0);
      const int64_t row0 = run.store_start + t0;
      int nvalid = 0;
      if (ok && nt > 0 && t_tile >= 0 && row0 >= 0) {
        const int64_t room = cap - row0;
        nvalid = room <= 0 ? 0 : (int)(room < nt ? room : nt);
      }
      if (ok && nt > 0 && nvalid < nt) bits |= MSHIFT_EBIT_STORE;
      if (nvalid > 0) {
        for (int t = lane; t < nt; t += 32) {
          int64_t slot;
          bool slot_ok = true;
          if (run.slots != nullptr) {
            slot = run.slots[t0 + t];
          } else {
            const int64_t pos = run.paged_start + t0 + t;
            const int64_t bi = pos >= 0 ? pos / a.block_size : -1;
            slot_ok = bi >= 0 && bi < run.block_table_len;
            slot = slot_ok ? (int64_t)run.block_table[bi] * a.block_size + pos % a.block_size : -1;
          }
          slot_ok = slot_ok && slot >= 0 && slot < a.num_slots;
          s_off[s][t] = (slot_ok && t < nvalid) ? (slot / a.block_size) * a.blk_stride +
                                                      (slot % a.block_size) * a.off_stride
                                                : -1;
          if (!slot_ok) atomicOr(a.err, MSHIFT_EBIT_SLOT);
        }
        if (HALF > 0 && tab != nullptr) {
          for (int i = lane; i < HALF; i += 32) {
            s_tab[s][i] = tab[i];
            s_tab[s][HALF + i] = tab[HALF + i];
          }
        }
      }
      if (lane == 0) {
        BulkMeta m;
        m.kbase = kbase;
        m.vbase = vbase;
        m.nt = nvalid > 0 ? nt : 0;
        m.rotate = (HALF > 0 && tab != nullptr) ? 1 : 0;
        s_meta[s] = m;
        if (bits) atomicOr(a.err, bits);
      }
      __syncwarp();  // the lanes' offsets and table are written before lane 0 publishes
      if (lane == 0) {
        if (nvalid > 0) {
          const uint32_t bytes = static_cast<uint32_t>(nvalid * row_bytes);
          mbar_expect_tx(&s_full[s], bytes);
          bulk_to_smem(s_data + s * stage_bytes, store + row0 * row_bytes, bytes, &s_full[s]);
        } else {
          mbar_arrive(&s_full[s]);
        }
      }
    }
    // Wait until every consumer warp has left its loop, then, if the launch
    // was aborted, for the copy last issued into each stage (the only one a
    // stage can still have in flight: a stage is refilled only after its
    // consumers released it), with the full bound and no abort shortcut, so
    // no copy is left writing shared memory when the CTA exits.
    cta_barrier_1(kBulkThreads);
    if (s_abort && lane == 0) {
      for (int kk = k - NS < 0 ? 0 : k - NS; kk < k; ++kk)
        (void)mbar_wait(&s_full[kk % NS], (kk / NS) & 1);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // e4m3 units carry twice the elements per byte: one unit in flight per
  // thread (MSHIFT_BULK_UNITS_E4M3 overrides), and the thread's cos/sin slice
  // held in registers for the whole stage.
  constexpr int U = E::kScaled ? kBulkUnitsE4m3 : 2;
  constexpr bool kRegTable = E::kScaled;
  const int g = threadIdx.x % G;
  const int u_first = threadIdx.x / G;
  const int ka = g < NP ? g : g + NP;
  const int kb = g < NP ? g + NP : g + G;
  for (int k = 0;; ++k) {
    const int s = k % NS;
    const uint32_t limit = (k == 0 && a.first_wait != 0u) ? a.first_wait - 1u : kWaitLimit;
    if (!warp_mbar_wait(&s_full[s], (k / NS) & 1, limit, &s_abort)) {
      if (lane == 0) atomicOr(a.err, MSHIFT_EBIT_TIMEOUT);
      s_abort = 1;
      break;
    }
    const BulkMeta m = s_meta[s];
    if (m.nt < 0) break;  // the producer's end-of-work stage
    const unsigned char* stage = s_data + s * stage_bytes;
    const int nu = m.nt * a.heads;
    const bool rotate = m.rotate && g < NP;
    float treg[kRegTable ? 2 * VEC : 4];
    const float* tc = s_tab[s] + g * VEC;
    const float* ts = s_tab[s] + HALF + g * VEC;
    if constexpr (kRegTable) {
      if (rotate) {
#pragma unroll
        for (int e = 0; e < VEC; e += 4) {
          *reinterpret_cast<float4*>(treg + e) = *reinterpret_cast<const float4*>(tc + e);
          *reinterpret_cast<float4*>(treg + VEC + e) = *reinterpret_cast<const float4*>(ts + e);
        }
      }
      tc = treg;
      ts = treg + VEC;
    }
    for (int u = u_first; u < nu; u += U * UPP) {
      Vec kv[U][2], vv[U][2];
      char* kp[U];
      char* vp[U];
      bool live[U];
#pragma unroll
      for (int q = 0; q < U; ++q) {
        const int uu = u + q * UPP;
        live[q] = false;
        if (uu < nu) {
          const int t = uu / a.heads;
          const int h = uu - t * a.heads;
          const int64_t off = s_off[s][t];
          if (off >= 0) {
            live[q] = true;
            const unsigned char* src = stage + (int64_t)uu * (2 * D * ES);
            kv[q][0] = lds_vec(src + ka * 16);
            kv[q][1] = lds_vec(src + kb * 16);
            vv[q][0] = lds_vec(src + D * ES + g * 16);
            vv[q][1] = lds_vec(src + D * ES + (g + G) * 16);
            kp[q] = m.kbase + (off + (int64_t)h * a.head_stride) * ES;
            vp[q] = m.vbase + (off + (int64_t)h * a.head_stride) * ES;
          }
        }
      }
#pragma unroll
      for (int q = 0; q < U; ++q) {
        if (!live[q]) continue;
        if (rotate) rotate_pair<E>(kv[q][0], kv[q][1], tc, ts);
        store_vec(kp[q] + ka * 16, kv[q][0]);
        store_vec(kp[q] + kb * 16, kv[q][1]);
        store_vec(vp[q] + g * 16, vv[q][0]);
        store_vec(vp[q] + (g + G) * 16, vv[q][1]);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&s_empty[s]);  // this warp is done reading stage s
  }
  cta_barrier_1(kBulkThreads);  // the producer drains after every consumer is out
}

// cos/sin of fp32(delta) * inv_freq[i], built exactly as the reference
// builds them on the GPU it serves from (src/marathon/shift_kernels.py:73-79:
// ``float(delta) * inv_freq`` in fp32, then torch's fp32 ``cos`` / ``sin`` on
// the cache's CUDA device, which are the CUDA math library's cosf / sinf):
// the angle is one fp32 product, then cosf and sinf.  With the reference's
// own tables the rotation that follows is the reference's, bit for bit.
__global__ void rope_tables_kernel(const int64_t* deltas, int32_t n, const float* inv_freq,
                                   int32_t half, float* out) {
  allow_dependents();  // the load kernel may launch; it waits for our writes
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < (int64_t)n * half) {
    const int64_t d = i / half;
    const int64_t j = i - d * half;
    const float ang = __fmul_rn(static_cast<float>(deltas[d]), inv_freq[j]);
    out[d * 2 * half + j] = cosf(ang);
    out[d * 2 * half + half + j] = sinf(ang);
  }
  // Launched as a programmatic dependent of the previous turn's load kernel,
  // this grid may run alongside it; it reads nothing that kernel writes, but
  // it must not complete before it, so that the next load kernel -- which
  // waits for this grid -- is ordered after the previous one too.
  wait_prior_grid();
}

// ------------------------------------------------------------------ dispatch
using KernelFn = void (*)(KArgs);
using BulkFn = void (*)(KArgs, int, int);

struct Variant {
  int32_t dtype, head_size, rotary;
  KernelFn load;
  KernelFn save;
  BulkFn bulk;
  int bulk_stages, bulk_stage_bytes, bulk_threads;
};

#define MSHIFT_VARIANT(E, DT, D, R)                                                    \
  {DT, D, R, move_kernel<E, D, R, false>, move_kernel<E, D, D, true>,                 \
   bulk_load_kernel<E, D, R>, bulk_stages<E>(), bulk_stage_bytes<E>(), bulk_threads<E>()}

const Variant kVariants[] = {
    MSHIFT_VARIANT(Bf16, MSHIFT_BF16, 128, 128),
    MSHIFT_VARIANT(Bf16, MSHIFT_BF16, 128, 64),
    MSHIFT_VARIANT(Bf16, MSHIFT_BF16, 64, 64),
    MSHIFT_VARIANT(Bf16, MSHIFT_BF16, 256, 256),
    MSHIFT_VARIANT(Bf16, MSHIFT_BF16, 256, 64),
    MSHIFT_VARIANT(F16, MSHIFT_F16, 128, 128),
    MSHIFT_VARIANT(F16, MSHIFT_F16, 64, 64),
    MSHIFT_VARIANT(F16, MSHIFT_F16, 256, 256),
    MSHIFT_VARIANT(F32, MSHIFT_F32, 128, 128),
    MSHIFT_VARIANT(E4m3, MSHIFT_E4M3, 128, 128),
    MSHIFT_VARIANT(E4m3, MSHIFT_E4M3, 256, 256),
};
constexpr int kNumVariants = sizeof(kVariants) / sizeof(kVariants[0]);

const Variant* find_variant(int32_t dtype, int32_t head_size, int32_t rotary, bool save) {
  for (const Variant& v : kVariants) {
    if (v.dtype != dtype || v.head_size != head_size) continue;
    if (save || v.rotary == rotary) return &v;
  }
  return nullptr;
}

thread_local char g_cuda_error[256] = "";

int cuda_fail(cudaError_t e) {
  std::snprintf(g_cuda_error, sizeof(g_cuda_error), "%s: %s", cudaGetErrorName(e),
                cudaGetErrorString(e));
  return MSHIFT_ECUDA;
}

// Persistent grid: SMs x resident CTAs of this kernel, cached per device.
struct GridCache {
  std::mutex mu;
  int sms[kMaxDevices] = {0};
  int occ[kMaxDevices][2 * kNumVariants] = {{0}};
  int bulk_smem[kMaxDevices][kNumVariants] = {{0}};  // dynamic smem the bulk kernel is set up for
  int bulk_occ[kMaxDevices][kNumVariants] = {{0}};
};
GridCache g_grid;

int grid_for(KernelFn fn, int variant_slot, int64_t total, int* grid) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return MSHIFT_EINVAL;
  std::lock_guard<std::mutex> lock(g_grid.mu);
  if (g_grid.sms[dev] == 0) {
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e);
    g_grid.sms[dev] = sms;
  }
  int& occ = g_grid.occ[dev][variant_slot];
  if (occ == 0) {
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kThreads, 0);
    if (e != cudaSuccess) return cuda_fail(e);
    if (occ < 1) occ = 1;
  }
  const int64_t cap = (int64_t)g_grid.sms[dev] * occ;
  *grid = static_cast<int>(total < cap ? total : cap);
  return MSHIFT_OK;
}

int check_paged(const mshift_paged* p) {
  if (p == nullptr) return MSHIFT_EINVAL;
  if (p->block_size <= 0 || p->heads <= 0 || p->head_size <= 0 || p->num_blocks < 0)
    return MSHIFT_EINVAL;
  if (p->blk_stride < 0 || p->off_stride < 0 || p->head_stride < 0) return MSHIFT_EINVAL;
  return MSHIFT_OK;
}

int elem_bytes(int32_t dtype) {
  switch (dtype) {
    case MSHIFT_BF16: case MSHIFT_F16: return 2;
    case MSHIFT_F32: return 4;
    case MSHIFT_E4M3: return 1;
    default: return 0;
  }
}

bool strides_aligned(int es, std::initializer_list<int64_t> strides) {
  for (int64_t s : strides)
    if ((s * es) % 16 != 0) return false;
  return true;
}

// Launch with programmatic stream serialization (see wait_prior_grid).
template <class... Params, class... Args>
cudaError_t launch_dependent(void (*fn)(Params...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, args...);
}

int launch(KernelFn fn, int slot, KArgs args, cudaStream_t stream, bool pdl = false) {
  const int64_t total = (int64_t)args.tiles_per_layer * args.n_layers;
  if (total <= 0) return MSHIFT_OK;
  int grid = 0;
  int st = grid_for(fn, slot, total, &grid);
  if (st != MSHIFT_OK) return st;
  // batched launches claim tiles dynamically while the claim counter fits
  // bits 8..31 of the status word
  args.dyn = (args.runs != nullptr && total + grid < (int64_t{1} << 24)) ? 1 : 0;
  cudaError_t e;
  if (pdl) {
    e = launch_dependent(fn, dim3(grid), dim3(kThreads), 0, stream, args);
  } else {
    fn<<<grid, kThreads, 0, stream>>>(args);
    e = cudaGetLastError();
  }
  return e == cudaSuccess ? MSHIFT_OK : cuda_fail(e);
}

int variant_slot(const Variant* v, bool save) {
  return static_cast<int>(v - kVariants) * 2 + (save ? 1 : 0);
}

// Which kernel serves loads: MSHIFT_KERNEL_LSU (128-bit loads), MSHIFT_KERNEL_BULK
// (TMA bulk copies through an mbarrier ring; used when the store rows are
// dense, else the LSU kernel runs) or MSHIFT_KERNEL_AUTO (the measured faster
// one on B200: TMA for e4m3, whose consumer warps are busy with the
// dequantise/requantise arithmetic, 128-bit loads for 16/32-bit types).
std::atomic<int> g_load_kernel{MSHIFT_KERNEL_AUTO};

// KArgs::first_wait of every batched load (0: normal waits); see
// mshift_debug_first_wait.
std::atomic<uint32_t> g_first_wait{0};

// Launch the TMA bulk load; returns MSHIFT_EUNSUPPORTED when the geometry does
// not fit a stage (the caller then uses the 128-bit-load kernel).
int launch_bulk(const Variant* v, const KArgs& args, int64_t row_bytes, cudaStream_t stream,
                bool pdl) {
  int part = static_cast<int>(v->bulk_stage_bytes / row_bytes);
  if (part > args.tile_tokens) part = args.tile_tokens;
  if (part > kBulkMaxPart) part = kBulkMaxPart;
  if (part < 1) return MSHIFT_EUNSUPPORTED;
  const int parts = (args.tile_tokens + part - 1) / part;
  const int64_t tiles = (int64_t)args.tiles_per_layer * args.n_layers;
  if (tiles * parts > INT32_MAX) return MSHIFT_EUNSUPPORTED;
  const int smem = static_cast<int>(v->bulk_stages * part * row_bytes);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return MSHIFT_EINVAL;
  const int vi = static_cast<int>(v - kVariants);
  int grid = 0;
  {
    std::lock_guard<std::mutex> lock(g_grid.mu);
    if (g_grid.sms[dev] == 0) {
      int sms = 0;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return cuda_fail(e);
      g_grid.sms[dev] = sms;
    }
    if (g_grid.bulk_smem[dev][vi] < smem) {
      e = cudaFuncSetAttribute(v->bulk, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return cuda_fail(e);
      int occ = 0;
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, v->bulk, v->bulk_threads, smem);
      if (e != cudaSuccess) return cuda_fail(e);
      if (occ < 1) return MSHIFT_EUNSUPPORTED;
      g_grid.bulk_smem[dev][vi] = smem;
      g_grid.bulk_occ[dev][vi] = occ;
    }
    // a CTA works through whole tiles, so more CTAs than tiles would idle
    const int64_t cap = (int64_t)g_grid.sms[dev] * g_grid.bulk_occ[dev][vi];
    grid = static_cast<int>(tiles < cap ? tiles : cap);
  }
  // tiles are claimed dynamically while the claim counter fits bits 8..31 of
  // the status word, as in the 128-bit-load kernel
  KArgs a = args;
  a.dyn = (a.runs != nullptr && tiles + grid < (int64_t{1} << 24)) ? 1 : 0;
  if (pdl) {
    e = launch_dependent(v->bulk, dim3(grid), dim3(v->bulk_threads), smem, stream, a, parts,
                         part);
  } else {
    v->bulk<<<grid, v->bulk_threads, smem, stream>>>(a, parts, part);
    e = cudaGetLastError();
  }
  return e == cudaSuccess ? MSHIFT_OK : cuda_fail(e);
}

int batched(bool save, const mshift_paged* paged, int32_t rotary, const mshift_run* runs,
            int32_t n_runs, int32_t tile_tokens, int32_t tiles_per_layer, int32_t n_layers,
            void* const* store_ptrs, const int64_t* store_caps, int32_t n_sessions, int64_t st_tok,
            int64_t st_head, void* const* k_ptrs, void* const* v_ptrs, const float* tables,
            int32_t n_tables, const float* k_scales, uint32_t* err, void* stream) {
  int st = check_paged(paged);
  if (st != MSHIFT_OK) return st;
  if (runs == nullptr || n_runs <= 0 || n_layers <= 0 || tiles_per_layer <= 0) return MSHIFT_EINVAL;
  if (tile_tokens <= 0 || tile_tokens > kMaxTile) return MSHIFT_EINVAL;
  if ((int64_t)tiles_per_layer * n_layers > INT32_MAX) return MSHIFT_EINVAL;
  if (store_ptrs == nullptr || store_caps == nullptr || n_sessions <= 0) return MSHIFT_EINVAL;
  if (k_ptrs == nullptr || v_ptrs == nullptr || err == nullptr) return MSHIFT_EINVAL;
  if (st_tok < 0 || st_head < 0) return MSHIFT_EINVAL;
  const int es = elem_bytes(paged->dtype);
  if (es == 0) return MSHIFT_EUNSUPPORTED;
  if (!strides_aligned(es, {paged->blk_stride, paged->off_stride, paged->head_stride, st_tok, st_head}))
    return MSHIFT_EINVAL;
  const Variant* v = find_variant(paged->dtype, paged->head_size, rotary, save);
  if (v == nullptr) return MSHIFT_EUNSUPPORTED;
  (void)k_scales;  // e4m3: the layer's K scale cancels (see rotate_word_e4m3)
  if (!save && n_tables > 0 && tables == nullptr) return MSHIFT_EINVAL;
  KArgs a{};
  a.runs = runs;
  a.n_runs = n_runs;
  a.tile_tokens = tile_tokens;
  a.tiles_per_layer = tiles_per_layer;
  a.n_layers = n_layers;
  a.store_ptrs = store_ptrs;
  a.store_caps = store_caps;
  a.n_sessions = n_sessions;
  a.block_size = paged->block_size;
  a.st_tok = st_tok;
  a.st_head = st_head;
  a.k_ptrs = k_ptrs;
  a.v_ptrs = v_ptrs;
  a.blk_stride = paged->blk_stride;
  a.off_stride = paged->off_stride;
  a.head_stride = paged->head_stride;
  a.num_slots = paged->num_blocks * paged->block_size;
  a.heads = paged->heads;
  a.n_tables = save ? 0 : n_tables;
  a.tables = save ? nullptr : tables;
  a.err = err;
  a.first_wait = g_first_wait.load(std::memory_order_relaxed);
  const int64_t row_elems = (int64_t)paged->heads * 2 * paged->head_size;
  const int kind = g_load_kernel.load(std::memory_order_relaxed);
  const bool want_bulk =
      kind == MSHIFT_KERNEL_BULK || (kind == MSHIFT_KERNEL_AUTO && paged->dtype == MSHIFT_E4M3);
  // a load with rotation tables normally follows the table kernel directly:
  // let its CTAs launch while that kernel finishes (they wait for its writes)
  const bool pdl = !save && n_tables > 0;
  if (!save && want_bulk && st_head == 2 * paged->head_size && st_tok == row_elems) {
    const int st = launch_bulk(v, a, row_elems * es, static_cast<cudaStream_t>(stream), pdl);
    if (st != MSHIFT_EUNSUPPORTED) return st;
  }
  return launch(save ? v->save : v->load, variant_slot(v, save), a,
                static_cast<cudaStream_t>(stream), pdl);
}

}  // namespace mshift

// ====================================================================== C ABI
using namespace mshift;

extern "C" {

int mshift_rope_tables(const int64_t* deltas, int32_t n, const float* inv_freq, int32_t half,
                       float* tables, void* stream) {
  if (n < 0 || half < 0) return MSHIFT_EINVAL;
  if (n == 0 || half == 0) return MSHIFT_OK;
  if (deltas == nullptr || inv_freq == nullptr || tables == nullptr) return MSHIFT_EINVAL;
  const int64_t total = (int64_t)n * half;
  const int threads = 128;
  const int64_t blocks = (total + threads - 1) / threads;
  if (blocks > INT32_MAX) return MSHIFT_EINVAL;
  const cudaError_t e = launch_dependent(rope_tables_kernel, dim3(static_cast<unsigned>(blocks)),
                                         dim3(threads), 0, static_cast<cudaStream_t>(stream),
                                         deltas, n, inv_freq, half, tables);
  return e == cudaSuccess ? MSHIFT_OK : cuda_fail(e);
}

int mshift_scatter_shifted(const void* src, int64_t src_tok_stride, int64_t src_head_stride,
                           int64_t n, void* k_base, void* v_base, const mshift_paged* paged,
                           const int64_t* slots, const float* table, int32_t rotary,
                           const float* k_scale, uint32_t* err, void* stream) {
  int st = check_paged(paged);
  if (st != MSHIFT_OK) return st;
  if (n < 0) return MSHIFT_EINVAL;
  if (n == 0) return MSHIFT_OK;  // zero-length load: nothing to do (shift_kernels.py:185-186)
  if (n > INT32_MAX) return MSHIFT_EINVAL;
  if (src == nullptr || k_base == nullptr || v_base == nullptr || slots == nullptr || err == nullptr)
    return MSHIFT_EINVAL;
  if (src_tok_stride < 0 || src_head_stride < 0) return MSHIFT_EINVAL;
  const int es = elem_bytes(paged->dtype);
  if (es == 0) return MSHIFT_EUNSUPPORTED;
  if (!strides_aligned(es, {paged->blk_stride, paged->off_stride, paged->head_stride,
                            src_tok_stride, src_head_stride}))
    return MSHIFT_EINVAL;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(k_base) |
       reinterpret_cast<uintptr_t>(v_base)) & 15u)
    return MSHIFT_EINVAL;
  const Variant* v = find_variant(paged->dtype, paged->head_size, rotary, false);
  if (v == nullptr) return MSHIFT_EUNSUPPORTED;
  (void)k_scale;  // e4m3: the layer's K scale cancels (see rotate_word_e4m3)
  const int32_t tt = mshift_default_tile_tokens(paged->heads);
  KArgs a{};
  a.runs = nullptr;
  a.n_runs = 1;
  a.tile_tokens = tt;
  a.tiles_per_layer = static_cast<int32_t>((n + tt - 1) / tt);
  a.n_layers = 1;
  a.n_sessions = 1;
  a.block_size = paged->block_size;
  a.st_tok = src_tok_stride;
  a.st_head = src_head_stride;
  a.blk_stride = paged->blk_stride;
  a.off_stride = paged->off_stride;
  a.head_stride = paged->head_stride;
  a.num_slots = paged->num_blocks * paged->block_size;
  a.heads = paged->heads;
  a.err = err;
  a.run0 = mshift_run{};
  a.run0.store_start = 0;
  a.run0.slots = slots;
  a.run0.len = static_cast<int32_t>(n);
  a.run0.table = table != nullptr ? 0 : -1;
  a.run0.tile_begin = 0;
  a.store0 = const_cast<void*>(src);
  a.cap0 = n;
  a.k0 = k_base;
  a.v0 = v_base;
  a.table0 = table;
  return launch(v->load, variant_slot(v, false), a, static_cast<cudaStream_t>(stream));
}

int mshift_load(const mshift_paged* paged, int32_t rotary, const mshift_run* runs, int32_t n_runs,
                int32_t tile_tokens, int32_t tiles_per_layer, int32_t n_layers,
                void* const* store_ptrs, const int64_t* store_caps, int32_t n_sessions,
                int64_t st_tok, int64_t st_head, void* const* k_ptrs, void* const* v_ptrs,
                const float* tables, int32_t n_tables, const float* k_scales, uint32_t* err,
                void* stream) {
  return batched(false, paged, rotary, runs, n_runs, tile_tokens, tiles_per_layer, n_layers,
                 store_ptrs, store_caps, n_sessions, st_tok, st_head, k_ptrs, v_ptrs, tables,
                 n_tables, k_scales, err, stream);
}

int mshift_save(const mshift_paged* paged, const mshift_run* runs, int32_t n_runs,
                int32_t tile_tokens, int32_t tiles_per_layer, int32_t n_layers,
                void* const* store_ptrs, const int64_t* store_caps, int32_t n_sessions,
                int64_t st_tok, int64_t st_head, void* const* k_ptrs, void* const* v_ptrs,
                uint32_t* err, void* stream) {
  return batched(true, paged, paged ? paged->head_size : 0, runs, n_runs, tile_tokens,
                 tiles_per_layer, n_layers, store_ptrs, store_caps, n_sessions, st_tok, st_head,
                 k_ptrs, v_ptrs, nullptr, 0, nullptr, err, stream);
}

int32_t mshift_plan_tiles(mshift_run* runs, int32_t n_runs, int32_t tile_tokens) {
  if (runs == nullptr || n_runs <= 0 || tile_tokens <= 0) return -1;
  int64_t acc = 0;
  for (int32_t i = 0; i < n_runs; ++i) {
    if (runs[i].len <= 0) return -1;
    runs[i].tile_begin = static_cast<int32_t>(acc);
    acc += (runs[i].len + tile_tokens - 1) / tile_tokens;
    if (acc > INT32_MAX) return -1;
  }
  return static_cast<int32_t>(acc);
}

int32_t mshift_default_tile_tokens(int32_t heads) {
  if (heads <= 0) return 16;
  int32_t t = 256 / heads;
  if (t < 16) t = 16;
  if (t > kMaxTile) t = kMaxTile;
  return t;
}

int mshift_supported(int32_t dtype, int32_t head_size, int32_t rotary) {
  return find_variant(dtype, head_size, rotary, false) != nullptr ? 1 : 0;
}

int mshift_set_load_kernel(int kind) {
  if (kind != MSHIFT_KERNEL_LSU && kind != MSHIFT_KERNEL_BULK && kind != MSHIFT_KERNEL_AUTO)
    return -1;
  return g_load_kernel.exchange(kind);
}

int32_t mshift_debug_first_wait(int32_t rounds) {
  const uint32_t prev = g_first_wait.exchange(rounds < 0 ? 0u : static_cast<uint32_t>(rounds) + 1u);
  return prev == 0u ? -1 : static_cast<int32_t>(prev - 1u);
}

const char* mshift_version(void) { return "marathon_b200 shift 0.1 (sm_100a)"; }

const char* mshift_strerror(int status) {
  switch (status) {
    case MSHIFT_OK: return "ok";
    case MSHIFT_EINVAL: return "invalid argument";
    case MSHIFT_EUNSUPPORTED: return "unsupported dtype / head_size / rotary combination";
    case MSHIFT_ECUDA: return "CUDA runtime error";
    case MSHIFT_ETOOBIG:
      return "request exceeds the static scratch of mshift_load_noalloc (256 deltas, rotary 256)";
    default: return "unknown status";
  }
}

const char* mshift_last_cuda_error(void) { return g_cuda_error; }

int mshift_stage(const mshift_copy* copies, int32_t n, void* stream) {
  if (n < 0 || (n > 0 && copies == nullptr)) return MSHIFT_EINVAL;
  for (int32_t i = 0; i < n; ++i) {
    const mshift_copy& c = copies[i];
    if (c.bytes < 0 || (c.bytes > 0 && (c.dst == nullptr || c.src == nullptr)))
      return MSHIFT_EINVAL;
  }
  auto s = static_cast<cudaStream_t>(stream);
  for (int32_t i = 0; i < n; ++i) {
    const mshift_copy& c = copies[i];
    if (c.bytes == 0) continue;
    cudaError_t e = cudaMemcpyAsync(c.dst, c.src, static_cast<size_t>(c.bytes),
                                    cudaMemcpyDefault, s);
    if (e != cudaSuccess) return cuda_fail(e);
  }
  return MSHIFT_OK;
}

int mshift_enable_peer(int32_t peer_device) {
  int cur = 0;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return cuda_fail(e);
  if (peer_device == cur) return MSHIFT_OK;
  int ok = 0;
  e = cudaDeviceCanAccessPeer(&ok, cur, peer_device);
  if (e != cudaSuccess) return cuda_fail(e);
  if (!ok) return MSHIFT_EUNSUPPORTED;
  e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();  // drop the recorded "already enabled" status
    return MSHIFT_OK;
  }
  return e == cudaSuccess ? MSHIFT_OK : cuda_fail(e);
}

}  // extern "C"

// ============================================ allocation-free batched load
//
// For callers that cannot allocate device memory: a process that must not
// call cudaMalloc once serving has started (a fixed memory budget handed out
// at start-up, a custom allocator owning the whole pool), or a host whose
// language binding can only pass pointers it already owns.  The batched load
// needs one piece of scratch between its two kernels, the rotation tables of
// the batch's deltas; here they live in a fixed array in the library's own
// device image, so the caller supplies only inputs and outputs.
//
// Limits: at most kNoAllocMaxTables distinct deltas per call and rotary/2 at
// most kNoAllocMaxHalf (256 x 2 x 128 floats = 256 KiB, held on every GPU that
// loads the library until the process exits).  Larger requests are rejected
// with MSHIFT_ETOOBIG before anything is launched.
//
// The array is shared by every call in the process: two calls whose work
// overlaps on the GPU (different streams, no ordering between them) race on
// it.  Nothing in it has to start at zero: each call's table kernel writes
// every row the following load kernel reads, in stream order.
//
// Set-up: the first call on a device, with that device current, resolves the
// array's device address with cudaGetSymbolAddress and caches it per device;
// that first call should come before any stream capture.

namespace mshift {
constexpr int kNoAllocMaxTables = 256;
constexpr int kNoAllocMaxHalf = 128;
}  // namespace mshift

static __device__ __align__(256) float
    g_noalloc_tables[mshift::kNoAllocMaxTables * 2 * mshift::kNoAllocMaxHalf];

namespace mshift {

struct NoAllocScratch {
  std::mutex mu;
  float* tables[kMaxDevices] = {nullptr};
};
NoAllocScratch g_noalloc;

// Device address of the scratch tables on the current device (set-up on first use).
int noalloc_tables(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return MSHIFT_EINVAL;
  std::lock_guard<std::mutex> lock(g_noalloc.mu);
  if (g_noalloc.tables[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_tables);
    if (e != cudaSuccess) return cuda_fail(e);
    g_noalloc.tables[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc.tables[dev];
  return MSHIFT_OK;
}

// The argument checks of the batched load, made before anything is launched.
int check_load_args(const mshift_paged* paged, int32_t rotary, const mshift_run* runs,
                    int32_t n_runs, int32_t tile_tokens, int32_t tiles_per_layer,
                    int32_t n_layers, void* const* store_ptrs, const int64_t* store_caps,
                    int32_t n_sessions, int64_t st_tok, int64_t st_head, void* const* k_ptrs,
                    void* const* v_ptrs, uint32_t* err) {
  int st = check_paged(paged);
  if (st != MSHIFT_OK) return st;
  if (runs == nullptr || n_runs <= 0 || n_layers <= 0 || tiles_per_layer <= 0) return MSHIFT_EINVAL;
  if (tile_tokens <= 0 || tile_tokens > kMaxTile) return MSHIFT_EINVAL;
  if ((int64_t)tiles_per_layer * n_layers > INT32_MAX) return MSHIFT_EINVAL;
  if (store_ptrs == nullptr || store_caps == nullptr || n_sessions <= 0) return MSHIFT_EINVAL;
  if (k_ptrs == nullptr || v_ptrs == nullptr || err == nullptr) return MSHIFT_EINVAL;
  if (st_tok < 0 || st_head < 0) return MSHIFT_EINVAL;
  const int es = elem_bytes(paged->dtype);
  if (es == 0) return MSHIFT_EUNSUPPORTED;
  if (!strides_aligned(es, {paged->blk_stride, paged->off_stride, paged->head_stride, st_tok, st_head}))
    return MSHIFT_EINVAL;
  if (find_variant(paged->dtype, paged->head_size, rotary, false) == nullptr)
    return MSHIFT_EUNSUPPORTED;
  return MSHIFT_OK;
}

}  // namespace mshift

extern "C" {

int mshift_load_noalloc(const mshift_paged* paged, int32_t rotary, const mshift_run* runs,
                        int32_t n_runs, int32_t tile_tokens, int32_t tiles_per_layer,
                        int32_t n_layers, void* const* store_ptrs, const int64_t* store_caps,
                        int32_t n_sessions, int64_t st_tok, int64_t st_head,
                        void* const* k_ptrs, void* const* v_ptrs, const int64_t* deltas,
                        int32_t n_deltas, const float* inv_freq, const float* k_scales,
                        uint32_t* err, void* stream) {
  if (n_deltas < 0 || rotary < 0 || (rotary & 1)) return MSHIFT_EINVAL;
  const int32_t half = rotary / 2;
  if (n_deltas > kNoAllocMaxTables || half > kNoAllocMaxHalf) return MSHIFT_ETOOBIG;
  if (n_deltas > 0 && (deltas == nullptr || inv_freq == nullptr)) return MSHIFT_EINVAL;
  int st = check_load_args(paged, rotary, runs, n_runs, tile_tokens, tiles_per_layer, n_layers,
                           store_ptrs, store_caps, n_sessions, st_tok, st_head, k_ptrs, v_ptrs,
                           err);
  if (st != MSHIFT_OK) return st;
  float* tables = nullptr;
  st = noalloc_tables(&tables);
  if (st != MSHIFT_OK) return st;
  if (n_deltas > 0) {
    st = mshift_rope_tables(deltas, n_deltas, inv_freq, half, tables, stream);
    if (st != MSHIFT_OK) return st;
  }
  return mshift_load(paged, rotary, runs, n_runs, tile_tokens, tiles_per_layer, n_layers,
                     store_ptrs, store_caps, n_sessions, st_tok, st_head, k_ptrs, v_ptrs,
                     n_deltas > 0 ? tables : nullptr, n_deltas, k_scales, err, stream);
}

int32_t mshift_noalloc_max_deltas(void) { return mshift::kNoAllocMaxTables; }

}  // extern "C"
