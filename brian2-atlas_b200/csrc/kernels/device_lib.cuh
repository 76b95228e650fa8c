// Device library prepended to every generated model translation unit (compiled
// by NVRTC for sm_100a with -fmad=false, so every a*b+c stays two IEEE
// roundings, as in the reference's non-fused CPU arithmetic).
//
// Contents:
//   * RunCtl: the per-run control block in device memory (tick cursor, error
//     word, spike-ring counters) that CUDA-graph-replayed kernels read.
//   * counter RNG (splitmix64 counters), restated from the reference
//     brian2-rust/src/executor.rs:190-336.
//   * Brian2 timestep() (brian2-rust/src/model.rs:981-992).
//   * ascending spike compaction: each tile stages its fired ids (warp ballot
//     + popc + block scan) and the last block of the launch lays the tiles
//     out in order, so a tick's spike list is globally ascending without any
//     block waiting on another;
//   * the GPU-to-GPU spike exchange (tagged 8-byte peer stores, bounded waits).
#pragma once

typedef unsigned long long u64;
typedef long long i64;
typedef unsigned int u32;
typedef int i32;
typedef unsigned short u16;
typedef unsigned char u8;

// Error bits OR-ed into RunCtl::error; the host maps them to messages.
#define B2_ERR_NONFINITE 0x1u
#define B2_ERR_TIMESTEP 0x2u
#define B2_ERR_BINOMIAL 0x4u
#define B2_ERR_POISSON 0x8u
#define B2_ERR_RING 0x10u
#define B2_ERR_LOOKBACK 0x20u
#define B2_ERR_INTDIV 0x40u
#define B2_ERR_TIMEDARRAY 0x80u
#define B2_ERR_CAST 0x100u
#define B2_ERR_EXCHANGE 0x200u
#define B2_ERR_BARRIER 0x400u

struct RunCtl {
  u64 tick_base;      // absolute tick of graph step k == 0
  u32 error;          // OR of B2_ERR_* bits
  u32 pad0;
  u64 reserved1;
  u64 reserved;
};

__device__ __forceinline__ double b2_bits(u64 r) { return __longlong_as_double((i64)r); }
__device__ __forceinline__ u64 b2_raw(double v) { return (u64)__double_as_longlong(v); }
// Exponent field not all ones (an integer test on the high word, which keeps
// the check off the FP64 pipe); the same answer as isfinite.
__device__ __forceinline__ bool b2_finite(double v) { return (__double2hiint(v) & 0x7ff00000) != 0x7ff00000; }

// ---------------------------------------------------------------- RNG
__device__ __forceinline__ u64 b2_mix64(u64 v) {
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}

// The draw's 53 random bits m; the uniform is exactly m * 2^-53.
__device__ __forceinline__ u64 b2_uniform_bits(u64 seed, u64 stream, u64 tick, u64 index, u64 draw) {
  u64 c = seed ^ (stream * 0x9e3779b97f4a7c15ull) ^ (tick * 0xd1b54a32d192ed03ull) ^
          (index * 0x94d049bb133111ebull) ^ (draw * 0x369dea0f31a53f85ull);
  return b2_mix64(c) >> 11;
}

__device__ __forceinline__ double b2_uniform_draw(u64 seed, u64 stream, u64 tick, u64 index, u64 draw) {
  return (double)b2_uniform_bits(seed, stream, tick, index, draw) * (1.0 / 9007199254740992.0);
}

__device__ __forceinline__ double b2_uniform(u64 seed, u64 stream, u64 tick, u64 index) {
  return b2_uniform_draw(seed, stream, tick, index, 0);
}

// Marsaglia polar method on pair index/2 (executor.rs:209-222).
__device__ double b2_normal(u64 seed, u64 stream, u64 tick, u64 index) {
  u64 pair = index >> 1;
  u64 draw = 0;
  for (int guard = 0; guard < 1 << 20; ++guard) {
    double x1 = 2.0 * b2_uniform_draw(seed, stream, tick, pair, draw) - 1.0;
    double x2 = 2.0 * b2_uniform_draw(seed, stream, tick, pair, draw + 1) - 1.0;
    double r = x1 * x1 + x2 * x2;
    if (r < 1.0 && r != 0.0) {
      double f = sqrt(-2.0 * log(r) / r);
      return f * ((index & 1) == 0 ? x1 : x2);
    }
    draw += 2;
  }
  return 0.0;
}

// Bring the line holding *p into this SM's L1 ahead of a dependent chain of
// loads (callers pass addresses the following code loads anyway).
__device__ __forceinline__ void b2_prefetch(const void* p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }

// ---------------------------------------------------------------- sorting
// In-place ascending sort of n keys by one thread: insertion sort for short
// runs (a target's events of one tick are usually a handful), heapsort
// (O(n log n), no recursion) beyond.
__device__ __forceinline__ void b2_sift_u64(u64* a, u32 root, u32 end) {
  while (2u * root + 1u < end) {
    u32 child = 2u * root + 1u;
    if (child + 1u < end && a[child] < a[child + 1u]) ++child;
    if (!(a[root] < a[child])) return;
    const u64 t = a[root];
    a[root] = a[child];
    a[child] = t;
    root = child;
  }
}

__device__ inline void b2_sort_u64(u64* a, u32 n) {
  if (n <= 16u) {
    for (u32 i = 1; i < n; ++i) {
      const u64 v = a[i];
      u32 j = i;
      while (j > 0u && a[j - 1u] > v) {
        a[j] = a[j - 1u];
        --j;
      }
      a[j] = v;
    }
    return;
  }
  for (u32 start = n / 2u; start-- > 0u;) b2_sift_u64(a, start, n);
  for (u32 end = n - 1u; end > 0u; --end) {
    const u64 t = a[0];
    a[0] = a[end];
    a[end] = t;
    b2_sift_u64(a, 0u, end);
  }
}

// Binomial inversion with the per-pathway constants precomputed on the host in
// glibc f64 (probability, q, q^n, restart bound), so the device loop is pure
// IEEE arithmetic and bit-identical to executor.rs:224-268.
__device__ double b2_binomial_inv(u64 seed, u64 stream, u64 tick, u64 index, u64 n,
                                  double probability, double q, double qn, double bound,
                                  bool reverse) {
  u64 draw = 0;
  for (int restarts = 0; restarts < 1 << 16; ++restarts) {
    u64 x = 0;
    double px = qn;
    double u = b2_uniform_draw(seed, stream, tick, index, draw);
    while (true) {
      if (u <= px) return (double)(reverse ? n - x : x);
      x += 1;
      if ((double)x > bound) {
        draw += 1;
        break;
      }
      u -= px;
      px = ((double)(n - x + 1) * probability * px) / ((double)x * q);
    }
  }
  return 0.0;
}

// The same inversion decided on the draw's integer bits: thr[x] is the
// largest m whose inversion returns at most x (host-built from the loop's
// own subtractions, non-decreasing), so the result is the number of
// thresholds below m, and K of them (m above every threshold) is a restart
// with the next draw.  The walk stops at the first threshold at or above m:
// the lanes still walking all read thr[x] at the same x (a broadcast), and
// no floating-point operation remains.
template <u32 K>
__device__ __forceinline__ double b2_binomial_thr(u64 seed, u64 stream, u64 tick, u64 index, u64 n,
                                                  const u64* __restrict__ thr, bool reverse) {
  for (u64 draw = 0; draw < (1ull << 16); ++draw) {
    const u64 m = b2_uniform_bits(seed, stream, tick, index, draw);
    u32 x = 0;
    while (x < K && m > thr[x]) ++x;
    if (x < K) return (double)(reverse ? n - x : x);
  }
  return 0.0;
}

// General binomial with a per-lane probability (device libm for q^n).
__device__ double b2_binomial(u64 seed, u64 stream, u64 tick, u64 index, u64 n, double p,
                              bool approximate) {
  if (p <= 0.0) return 0.0;
  if (p >= 1.0) return (double)n;
  double nf = (double)n;
  double loc = nf * p;
  double complement = nf * (1.0 - p);
  if (approximate && loc > 5.0 && complement > 5.0)
    return b2_normal(seed, stream, tick, index) * sqrt(loc * (1.0 - p)) + loc;
  bool reverse = p > 0.5;
  double probability = reverse ? 1.0 - p : p;
  double q = 1.0 - probability;
  double qn = exp(nf * log(q));
  double bound = fmin(nf, nf * probability + 10.0 * sqrt(nf * probability * q + 1.0));
  return b2_binomial_inv(seed, stream, tick, index, n, probability, q, qn, bound, reverse);
}

__device__ double b2_log_gamma_positive(double value) {
  const double c[8] = {676.5203681218851,    -1259.1392167224028, 771.3234287776531,
                       -176.6150291621406,   12.507343278686905,  -0.13857109526572012,
                       9.984369578019572e-6, 1.5056327351493116e-7};
  double z = value - 1.0;
  double x = 0.9999999999998099;
  for (int i = 0; i < 8; ++i) x += c[i] / (z + (double)i + 1.0);
  double t = z + 7.5;
  return 0.9189385332046727 + (z + 0.5) * log(t) - t + log(x);
}

// Knuth product below 10, Hoermann PTRS above (executor.rs:290-336).
__device__ double b2_poisson(u64 seed, u64 stream, u64 tick, u64 index, double lambda) {
  if (lambda == 0.0) return 0.0;
  if (!isfinite(lambda) || !(lambda >= 0.0 && lambda <= 1.0e12)) return __longlong_as_double(0x7ff8000000000000ll);
  if (lambda < 10.0) {
    double limit = exp(-lambda);
    double product = 1.0;
    for (u64 sample = 0; sample < (1ull << 24); ++sample) {
      product *= b2_uniform_draw(seed, stream, tick, index, sample);
      if (product <= limit) return (double)sample;
    }
    return 0.0;
  }
  double root = sqrt(lambda);
  double b = 0.931 + 2.53 * root;
  double a = -0.059 + 0.02483 * b;
  double inverse_alpha = 1.1239 + 1.1328 / (b - 3.4);
  double squeeze = 0.9277 - 3.6224 / (b - 2.0);
  u64 draw = 0;
  for (int guard = 0; guard < 1 << 20; ++guard) {
    double u = b2_uniform_draw(seed, stream, tick, index, draw) - 0.5;
    double v = b2_uniform_draw(seed, stream, tick, index, draw + 1);
    draw += 2;
    double us = 0.5 - fabs(u);
    double candidate = floor((2.0 * a / us + b) * u + lambda + 0.43);
    if (us >= 0.07 && v <= squeeze) return candidate;
    if (candidate < 0.0 || (us < 0.013 && v > us)) continue;
    double left = log(v * inverse_alpha / (a / (us * us) + b));
    double right = -lambda + candidate * log(lambda) - b2_log_gamma_positive(candidate + 1.0);
    if (left <= right) return candidate;
  }
  return 0.0;
}

// Brian2 timestep(): floor((t + 1e-3 dt) / dt) with range checks.
__device__ __forceinline__ u64 b2_timestep(double time, double dt, u32& err) {
  double steps = (time + 1e-3 * dt) / dt;
  if (!(time >= 0.0 && isfinite(dt) && dt > 0.0 && isfinite(steps) && steps < 9223372036854775808.0)) {
    err |= B2_ERR_TIMESTEP;
    return 0;
  }
  return (u64)steps;
}

__device__ __forceinline__ double b2_timestep_reg(double time, double dt, u32& err) {
  u64 v = b2_timestep(time, dt, err);
  if (v > 9007199254740992ull) {
    err |= B2_ERR_TIMESTEP;
    return 0.0;
  }
  return (double)v;
}

__device__ __forceinline__ double b2_binomial_checked(u64 seed, u64 stream, u64 tick, u64 index, u64 n,
                                                      double p, bool approximate, u32& err) {
  if (!(isfinite(p) && p >= 0.0 && p <= 1.0)) {
    err |= B2_ERR_BINOMIAL;
    return 0.0;
  }
  return b2_binomial(seed, stream, tick, index, n, p, approximate);
}

// ---------------------------------------------------------------- TimedArray
// Op::TimedArray (executor.rs:6121-6154): row = trunc((t / epsilon + 0.5) /
// upsampling) clamped to [0, rows - 1] (a NaN row is row 0, like Rust's
// saturating cast); with columns, the index must be finite and in
// [0, width); a bad index or a non-finite value sets B2_ERR_TIMEDARRAY.
__device__ __forceinline__ double b2_timed_array(const double* __restrict__ values, u64 rows, u64 width,
                                                 bool has_columns, double epsilon, double upsampling, double time,
                                                 double column, u32& err) {
  const double raw_row = trunc((time / epsilon + 0.5) / upsampling);
  const u64 row = !(raw_row > 0.0) ? 0ull : (raw_row >= (double)(rows - 1) ? rows - 1 : (u64)raw_row);
  u64 col = 0;
  if (has_columns) {
    if (!(isfinite(column) && column >= 0.0 && column < (double)width)) {
      err |= B2_ERR_TIMEDARRAY;
      return 0.0;
    }
    col = (u64)column;
  }
  return values[row * width + col];
}

// ---------------------------------------------------------------- scalar ops

// Per-op rules of the reference evaluate() (executor.rs:5932-6158).
__device__ __forceinline__ double b2_exprel(double a) {
  if (fabs(a) < 1e-16) return 1.0;
  if (a > 717.0) return __longlong_as_double(0x7ff0000000000000ll);
  return expm1(a) / a;
}
__device__ __forceinline__ double b2_trunc(double a) {
  return fabs(a) <= 9007199254740992.0 ? trunc(a) : __longlong_as_double(0x7ff8000000000000ll);
}
__device__ __forceinline__ double b2_round_f32(double a) {
  float f = (float)a;
  return isfinite(f) ? (double)f : __longlong_as_double(0x7ff8000000000000ll);
}
__device__ __forceinline__ double b2_fmod_floor(double a, double b) { return a - b * floor(a / b); }
__device__ __forceinline__ double b2_tick_offset(double a, i64 offset) {
  double r = a + (double)offset;
  return fabs(r) <= 9007199254740992.0 ? r : __longlong_as_double(0x7ff8000000000000ll);
}

// ---------------------------------------------------------------- casts
// Rust `as` float -> int casts saturate and send NaN to 0.
__device__ __forceinline__ i64 b2_f2i64(double x) {
  if (isnan(x)) return 0;
  if (x <= -9223372036854775808.0) return (i64)0x8000000000000000ull;
  if (x >= 9223372036854775808.0) return 0x7fffffffffffffffll;
  return (i64)x;
}
__device__ __forceinline__ u64 b2_f2u64(double x) {
  if (isnan(x) || x <= 0.0) return 0;
  if (x >= 18446744073709551616.0) return 0xffffffffffffffffull;
  return (u64)x;
}
__device__ __forceinline__ i32 b2_f2i32(double x) {
  i64 v = b2_f2i64(x);
  return v < -2147483648ll ? (i32)0x80000000u : v > 2147483647ll ? 2147483647 : (i32)v;
}
__device__ __forceinline__ u32 b2_f2u32(double x) {
  u64 v = b2_f2u64(x);
  return v > 0xffffffffull ? 0xffffffffu : (u32)v;
}

template <class T>
__device__ __forceinline__ T b2_floor_mod(T a, T b) {
  T q = a / b, r = a % b;
  T fq = (r != 0 && ((r < 0) != (b < 0))) ? (T)(q - 1) : q;
  return (T)(a - fq * b);
}
template <class T>
__device__ __forceinline__ T b2_floor_div(T a, T b) {
  T q = a / b, r = a % b;
  return (r != 0 && ((r < 0) != (b < 0))) ? (T)(q - 1) : q;
}

// Integer register ops (integer_unary_value / integer_binary_value,
// executor.rs:5831-5930).  dtype: 0 i32, 1 i64, 2 u32, 3 u64; op: 0 add,
// 1 sub, 2 mul, 3 floor-mod, 4 floor-div, 5 gt, 6 ge, 7 lt, 8 le.
__device__ __forceinline__ double b2_int_neg(int dtype, double a) {
  u64 r = b2_raw(a);
  return dtype == 0 ? b2_bits((u64)(u32)(0u - (u32)r)) : b2_bits(0ull - r);
}
__device__ __forceinline__ double b2_int_abs(int dtype, double a) {
  u64 r = b2_raw(a);
  if (dtype == 0) {
    i32 v = (i32)(u32)r;
    return b2_bits((u64)(v < 0 ? (0u - (u32)v) : (u32)v));
  }
  i64 v = (i64)r;
  return b2_bits(v < 0 ? 0ull - (u64)v : (u64)v);
}
template <class S, class U>
__device__ __forceinline__ double b2_int_signed(int op, S a, S b, S minv, u32& err, bool narrow) {
  u64 out;
  switch (op) {
    case 5: return a > b ? 1.0 : 0.0;
    case 6: return a >= b ? 1.0 : 0.0;
    case 7: return a < b ? 1.0 : 0.0;
    case 8: return a <= b ? 1.0 : 0.0;
    case 0: out = (u64)(U)((U)a + (U)b); break;
    case 1: out = (u64)(U)((U)a - (U)b); break;
    case 2: out = (u64)(U)((U)a * (U)b); break;
    case 3:
      if (b == 0) { err |= B2_ERR_INTDIV; return 0.0; }
      out = (u64)(U)((a == minv && b == (S)-1) ? (S)0 : b2_floor_mod<S>(a, b));
      break;
    default:
      if (b == 0) { err |= B2_ERR_INTDIV; return 0.0; }
      out = (u64)(U)((a == minv && b == (S)-1) ? minv : b2_floor_div<S>(a, b));
      break;
  }
  return b2_bits(narrow ? (u64)(u32)out : out);
}
template <class U>
__device__ __forceinline__ double b2_int_unsigned(int op, U a, U b, u32& err) {
  switch (op) {
    case 5: return a > b ? 1.0 : 0.0;
    case 6: return a >= b ? 1.0 : 0.0;
    case 7: return a < b ? 1.0 : 0.0;
    case 8: return a <= b ? 1.0 : 0.0;
    case 0: return b2_bits((u64)(U)(a + b));
    case 1: return b2_bits((u64)(U)(a - b));
    case 2: return b2_bits((u64)(U)(a * b));
    case 3:
      if (b == 0) { err |= B2_ERR_INTDIV; return 0.0; }
      return b2_bits((u64)(a % b));
    default:
      if (b == 0) { err |= B2_ERR_INTDIV; return 0.0; }
      return b2_bits((u64)(a / b));
  }
}
__device__ __forceinline__ double b2_int_binary(int dtype, int op, double a, double b, u32& err) {
  u64 x = b2_raw(a), y = b2_raw(b);
  switch (dtype) {
    case 0: return b2_int_signed<i32, u32>(op, (i32)(u32)x, (i32)(u32)y, (i32)0x80000000u, err, true);
    case 1: return b2_int_signed<i64, u64>(op, (i64)x, (i64)y, (i64)0x8000000000000000ull, err, false);
    case 2: return b2_int_unsigned<u32>(op, (u32)x, (u32)y, err);
    default: return b2_int_unsigned<u64>(op, x, y, err);
  }
}

// ---------------------------------------------------------------- atomics
// f32 state commit `(float)((double)old + add)`, applied as one atomic step.
// Every event of a constant-weight pathway applies the same map, so the final
// value is independent of the order in which the updates land.
// Returns false when the rounded result is not finite (the reference raises).
__device__ __forceinline__ bool b2_atomic_add_f32_via_f64(float* addr, double add) {
  u32* a = (u32*)addr;
  u32 old = *((volatile u32*)a), assumed;
  float next;
  do {
    assumed = old;
    next = (float)((double)__uint_as_float(assumed) + add);
    old = atomicCAS(a, assumed, __float_as_uint(next));
  } while (old != assumed);
  return isfinite(next);
}

// ---------------------------------------------------------------- block scan
// Exclusive prefix of one u32 per thread over a block of THREADS threads;
// *total receives the block sum (every thread).
template <int THREADS>
__device__ __forceinline__ u32 b2_block_exclusive_scan(u32 v, u32* total) {
  __shared__ u32 s_part[THREADS / 32 + 1];
  const u32 lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  u32 x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    u32 y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= (u32)d) x += y;
  }
  if (lane == 31) s_part[warp] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    u32 acc = 0;
    for (int w = 0; w < THREADS / 32; ++w) {
      u32 c = s_part[w];
      s_part[w] = acc;
      acc += c;
    }
    s_part[THREADS / 32] = acc;
  }
  __syncthreads();
  *total = s_part[THREADS / 32];
  const u32 r = s_part[warp] + x - v;
  __syncthreads();  // s_part may be reused by the next call
  return r;
}

// ---------------------------------------------------------------- GPU-to-GPU spike exchange
// Every rank owns a contiguous block of each population and publishes the
// tick's ascending list of its block's spikes (global ids) to every rank,
// itself included: one aligned 8-byte store {value, tag} per id, plus one
// {count, tag} word, into the receiver's inbox through a CUDA IPC mapping
// over NVLink.  An aligned 8-byte store is single-copy atomic, so a receiver
// that reads the tag of the current tick also reads that tick's value: no
// fence and no separate ready flag are needed (the "low-latency" protocol of
// NVIDIA's collective library).  Inbox layout per parity half: rank q's slot
// starts at word q + lo_q (lo_q = first neuron of q's block): its count word,
// then up to (block size) id words.  The two halves are used on alternate
// ticks; a rank cannot run two ticks ahead of a peer, because its own tick t+1
// needs the peer's list of tick t+1, which the peer only publishes after it
// has consumed tick t.
__device__ __forceinline__ void b2_ll_store(u64* p, u32 word, u32 tag) {
  const u64 v = ((u64)tag << 32) | (u64)word;
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ u64 b2_ll_load(const u64* p) {
  u64 v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ u64 b2_globaltimer() {
  u64 t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Word of the current tick at p.  The wait is bounded twice: by the global
// timer (timeout_ns) and by an iteration count; on expiry it records
// B2_ERR_EXCHANGE and returns 0, so the kernel ends and the host sees the error.
__device__ __forceinline__ u32 b2_ll_wait(const u64* p, u32 tag, u64 timeout_ns, u32& err) {
  u64 v = b2_ll_load(p);
  if ((u32)(v >> 32) == tag) return (u32)v;
  const u64 t0 = b2_globaltimer();
  for (u64 it = 0; it < (1ull << 28); ++it) {
    __nanosleep(32);
    v = b2_ll_load(p);
    if ((u32)(v >> 32) == tag) return (u32)v;
    if ((it & 15) == 0 && b2_globaltimer() - t0 > timeout_ns) break;
  }
  err |= B2_ERR_EXCHANGE;
  return 0u;
}

// L2 eviction priorities for a scatter: row entries are read once per tick
// (evict first), the per-target counters they index are reused by every
// event (evict last).
__device__ __forceinline__ u64 b2_policy_evict_first() {
  u64 pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ u64 b2_policy_evict_last() {
  u64 pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// Build-time data only (the read-only path).
__device__ __forceinline__ u32 b2_ld_rows(const u32* p, u64 pol) {
  u32 v;
  asm volatile("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol));
  return v;
}
__device__ __forceinline__ void b2_red_add_hint(u32* p, u32 v, u64 pol) {
  asm volatile("red.global.add.L2::cache_hint.u32 [%0], %1, %2;" ::"l"(p), "r"(v), "l"(pol) : "memory");
}

// Grid-wide barrier of a co-resident (cooperatively launched) grid: every
// block adds one arrival to *bar and waits until *bar reaches `target` (the
// barriers passed so far times the grid's blocks).  The arrival is a release
// (fence, then the add) and the wait an acquire, so everything any block
// wrote before the barrier is visible to every block after it.  Bounded like
// the exchange waits: on expiry a block stops waiting and the run reports the
// error, and once one barrier has expired no later barrier waits.
__device__ __forceinline__ void b2_grid_barrier(u32* bar, u32 target, RunCtl* ctl, u64 timeout_ns) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
    u32 v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
    if (v < target) {
      const u64 t0 = b2_globaltimer();
      for (u64 it = 0; it < (1ull << 28); ++it) {
        __nanosleep(32);
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
        if (v >= target) break;
        if ((it & 15) == 0 &&
            (b2_globaltimer() - t0 > timeout_ns || (*(volatile const u32*)&ctl->error & B2_ERR_BARRIER) != 0u)) {
          atomicOr(&ctl->error, B2_ERR_BARRIER);
          break;
        }
      }
      if (v < target) atomicOr(&ctl->error, B2_ERR_BARRIER);
    }
    __threadfence();
  }
  __syncthreads();
}

// Exclusive offsets of the tiles' staged counts for the calling thread's
// contiguous tile range [*t0, *t1) (the last block of a step launch; every
// tile's count is visible): *pos = spikes before the range, *total = all.
template <int THREADS>
__device__ __forceinline__ void b2_tile_offsets(u32 tiles, const u32* tile_count, u32* t0, u32* t1, u32* pos,
                                                u32* total) {
  __shared__ u32 s_warp_sum[THREADS / 32];
  __shared__ u32 s_total;
  const u32 per = (tiles + THREADS - 1) / THREADS;
  *t0 = threadIdx.x * per;
  *t1 = min(tiles, *t0 + per);
  u32 mine = 0;
  for (u32 t = *t0; t < *t1; ++t) mine += __ldcg(tile_count + t);
  const u32 lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  u32 x = mine;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    u32 y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= (u32)d) x += y;
  }
  if (lane == 31) s_warp_sum[warp] = x;
  __syncthreads();
  if (threadIdx.x == 0) {
    u32 acc = 0;
    for (int w = 0; w < THREADS / 32; ++w) {
      u32 c = s_warp_sum[w];
      s_warp_sum[w] = acc;
      acc += c;
    }
    s_total = acc;
  }
  __syncthreads();
  *pos = s_warp_sum[warp] + (x - mine);
  *total = s_total;
}

// Lay out a tick's staged spike ids: every tile staged its ascending ids at
// stage[tile * tile_n ...] and its count at tile_count[tile]; the last block
// of the launch (after all tiles' stores are visible) computes the tiles'
// exclusive offsets and copies the ids into the ring in tile order, which is
// ascending neuron order.  Writes tick_start[rel + 1].
template <int THREADS>
__device__ void b2_finalize_spikes(u32 tiles, u32 tile_n, const u32* tile_count, const u32* stage, u32* ring,
                                   u64 mask, u64* tick_start, u64 rel, u64 cap, u64 floor, u32& err) {
  u32 t0, t1, off, total;
  b2_tile_offsets<THREADS>(tiles, tile_count, &t0, &t1, &off, &total);
  const u64 base = tick_start[rel];
  u64 pos = base + off;
  for (u32 t = t0; t < t1; ++t) {
    const u32 n = __ldcg(tile_count + t);
    for (u32 k = 0; k < n; ++k) ring[(pos + k) & mask] = __ldcg(stage + (u64)t * tile_n + k);
    pos += n;
  }
  if (threadIdx.x == 0) {
    const u64 end = base + total;
    tick_start[rel + 1] = end;
    if (end - floor > cap) err |= B2_ERR_RING;
  }
}
