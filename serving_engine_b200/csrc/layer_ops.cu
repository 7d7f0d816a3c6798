// Decode-layer glue fused around the attention path for the tensor-parallel
// decoder: RoPE + KV append, residual add + RMSNorm, SwiGLU.
//
// seb_rope_kv_append folds the rotary embedding (HF apply_rotary_pos_emb, the
// rotate-half form) into the KV write of _PagedKVCache.write
// (serving_engine/model_runner.py:21-32): the qkv projection's output is read
// once, q is written rotated for the attention call, rotated K and V go straight
// to their slot_mapping positions. Products and sums are rounded to the 16-bit
// type exactly as the eager `x * cos + rotate_half(x) * sin` rounds them, so the
// result is bit-identical to the unfused torch ops.
//
// seb_add_rmsnorm and seb_swiglu replace the residual add + RMSNorm pair and
// silu(gate) * up of each decoder layer; they compute in fp32 and round once.
//
// Roofline: HBM (a few MB per call); at decode sizes these are launch-latency
// bound, which is what fusing them saves.
#include "seb_common.cuh"
#include "seb_vec.cuh"

#include <algorithm>

namespace seb {
namespace {

template <typename T>
__device__ __forceinline__ float f32(T x) {
  return Elem<T>::to_float(x);
}
template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return Elem<T>::to_float(Elem<T>::from_float(x));
}

struct RopeParams {
  const char* qkv;
  int64_t qkv_st;  // bytes per token
  const char* cos;
  const char* sin;
  int64_t cs_st;  // bytes per token
  const int64_t* slots;
  int64_t num_slots;
  char* q_out;
  int64_t q_st;  // bytes per token; heads contiguous
  char* k_cache;
  char* v_cache;
  int64_t n_tokens;
  int32_t hq, hkv, d;
  int32_t pairs;  // 1: 4-byte element-pair accesses are aligned
  int32_t* err;
};

// One warp per (token, row): rows [0, hq) are q heads, [hq, hq + hkv) k heads,
// [hq + hkv, hq + 2 hkv) v heads of the token's qkv vector.
template <typename T>
__global__ void __launch_bounds__(256) rope_append_kernel(RopeParams p) {
  const int64_t w = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int rows = p.hq + 2 * p.hkv;
  const int64_t t = w / rows;
  const int r = (int)(w % rows);
  if (t >= p.n_tokens) return;
  const T* src = reinterpret_cast<const T*>(p.qkv + t * p.qkv_st) + (int64_t)r * p.d;
  T* dst;
  if (r < p.hq) {
    dst = reinterpret_cast<T*>(p.q_out + t * p.q_st) + (int64_t)r * p.d;
  } else {
    const int64_t slot = __ldg(p.slots + t);
    if (slot < 0 || slot >= p.num_slots) {
      if (lane == 0 && r == p.hq) atomic_or_err(p.err, SEB_ERRBIT_SLOT);
      return;
    }
    const bool is_v = r >= p.hq + p.hkv;
    const int h = (r - p.hq) - (is_v ? p.hkv : 0);
    dst = reinterpret_cast<T*>(is_v ? p.v_cache : p.k_cache) + (slot * p.hkv + h) * p.d;
    if (is_v) {
      if (p.pairs) {
        for (int i = 2 * lane; i < p.d; i += 64)
          *reinterpret_cast<uint32_t*>(dst + i) = *reinterpret_cast<const uint32_t*>(src + i);
      } else {
        for (int i = lane; i < p.d; i += 32) dst[i] = src[i];
      }
      return;
    }
  }
  const T* cs = reinterpret_cast<const T*>(p.cos + t * p.cs_st);
  const T* sn = reinterpret_cast<const T*>(p.sin + t * p.cs_st);
  const int half = p.d / 2;
  if (p.pairs) {
    // element pairs: 4-byte accesses (head_dim % 4 == 0, rows 4-byte aligned)
    using P2 = uint32_t;
    for (int i = 2 * lane; i < half; i += 64) {
      const P2 x1p = *reinterpret_cast<const P2*>(src + i), x2p = *reinterpret_cast<const P2*>(src + i + half);
      const P2 c1p = *reinterpret_cast<const P2*>(cs + i), c2p = *reinterpret_cast<const P2*>(cs + i + half);
      const P2 s1p = *reinterpret_cast<const P2*>(sn + i), s2p = *reinterpret_cast<const P2*>(sn + i + half);
      const T* x1 = reinterpret_cast<const T*>(&x1p);
      const T* x2 = reinterpret_cast<const T*>(&x2p);
      const T* c1 = reinterpret_cast<const T*>(&c1p);
      const T* c2 = reinterpret_cast<const T*>(&c2p);
      const T* s1 = reinterpret_cast<const T*>(&s1p);
      const T* s2 = reinterpret_cast<const T*>(&s2p);
      P2 lo, hi;
      T* lo_e = reinterpret_cast<T*>(&lo);
      T* hi_e = reinterpret_cast<T*>(&hi);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float a = f32(x1[e]), b = f32(x2[e]);
        lo_e[e] = Elem<T>::from_float(round_to<T>(a * f32(c1[e])) + round_to<T>(-b * f32(s1[e])));
        hi_e[e] = Elem<T>::from_float(round_to<T>(b * f32(c2[e])) + round_to<T>(a * f32(s2[e])));
      }
      *reinterpret_cast<P2*>(dst + i) = lo;
      *reinterpret_cast<P2*>(dst + i + half) = hi;
    }
    return;
  }
  for (int i = lane; i < half; i += 32) {
    const float x1 = f32(src[i]), x2 = f32(src[i + half]);
    // rotate_half(x) = (-x2, x1); each product and the sum rounded like the eager ops
    const float lo = round_to<T>(x1 * f32(cs[i])) + round_to<T>(-x2 * f32(sn[i]));
    const float hi = round_to<T>(x2 * f32(cs[i + half])) + round_to<T>(x1 * f32(sn[i + half]));
    dst[i] = Elem<T>::from_float(lo);
    dst[i + half] = Elem<T>::from_float(hi);
  }
}

// rope_append_kernel with 16-byte accesses (every row and table 16-byte aligned,
// head_dim % 16 == 0): one thread per (token, 8-element chunk). A q or k row is
// head_dim / 16 threads, each rotating elements [i, i + 8) with [i + half,
// i + half + 8); a v row is head_dim / 8 threads, each copying one chunk. The
// per-element arithmetic is the one of rope_append_kernel, so both give the
// same bits; a token's hundreds of threads keep all of its loads in flight at
// once, where one warp per row left half its lanes idle at head_dim 64.
template <typename T>
__global__ void __launch_bounds__(256) rope_append_vec_kernel(RopeParams p) {
  const int ch = p.d >> 4;  // chunks in half a row
  const int rot_threads = (p.hq + p.hkv) * ch;
  const int per_token = rot_threads + p.hkv * 2 * ch;
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t t = g / per_token;
  if (t >= p.n_tokens) return;
  const int rem = (int)(g - t * per_token);
  const T* src_tok = reinterpret_cast<const T*>(p.qkv + t * p.qkv_st);
  if (rem >= rot_threads) {  // v: copy one chunk into the token's slot
    const int r2 = rem - rot_threads;
    const int h = r2 / (2 * ch), c = r2 - h * 2 * ch;
    const int64_t slot = __ldg(p.slots + t);
    if (slot < 0 || slot >= p.num_slots) return;  // reported by the k rows
    const uint4 v = *reinterpret_cast<const uint4*>(src_tok + (int64_t)(p.hq + p.hkv + h) * p.d + 8 * c);
    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.v_cache) + (slot * p.hkv + h) * p.d + 8 * c) = v;
    return;
  }
  const int r = rem / ch, c = rem - r * ch;
  const int half = p.d >> 1;
  const int i = 8 * c;
  T* dst;
  if (r < p.hq) {
    dst = reinterpret_cast<T*>(p.q_out + t * p.q_st) + (int64_t)r * p.d;
  } else {
    const int64_t slot = __ldg(p.slots + t);
    if (slot < 0 || slot >= p.num_slots) {
      if (r == p.hq && c == 0) atomic_or_err(p.err, SEB_ERRBIT_SLOT);
      return;
    }
    dst = reinterpret_cast<T*>(p.k_cache) + (slot * p.hkv + (r - p.hq)) * p.d;
  }
  const T* src = src_tok + (int64_t)r * p.d;
  const T* cs = reinterpret_cast<const T*>(p.cos + t * p.cs_st);
  const T* sn = reinterpret_cast<const T*>(p.sin + t * p.cs_st);
  Vec8<T> x1, x2, c1, c2, s1, s2, lo, hi;
  x1.raw = *reinterpret_cast<const uint4*>(src + i);
  x2.raw = *reinterpret_cast<const uint4*>(src + i + half);
  c1.raw = __ldg(reinterpret_cast<const uint4*>(cs + i));
  c2.raw = __ldg(reinterpret_cast<const uint4*>(cs + i + half));
  s1.raw = __ldg(reinterpret_cast<const uint4*>(sn + i));
  s2.raw = __ldg(reinterpret_cast<const uint4*>(sn + i + half));
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float a = x1.get(e), b = x2.get(e);
    lo.set(e, round_to<T>(a * c1.get(e)) + round_to<T>(-b * s1.get(e)));
    hi.set(e, round_to<T>(b * c2.get(e)) + round_to<T>(a * s2.get(e)));
  }
  *reinterpret_cast<uint4*>(dst + i) = lo.raw;
  *reinterpret_cast<uint4*>(dst + i + half) = hi.raw;
}

// One CTA per row: x <- round(x + a) (when a is given), out = x * rsqrt(mean(x^2) + eps) * w.
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS) add_rmsnorm_kernel(T* x, int64_t x_st, const T* a, int64_t a_st,
                                                              const T* w, T* out, int64_t o_st, int hidden,
                                                              float eps) {
  constexpr int kMaxPerThread = 32;
  __shared__ float red[THREADS / 32];
  const int64_t row = blockIdx.x;
  T* xr = x + row * x_st;
  const T* ar = a ? a + row * a_st : nullptr;
  float v[kMaxPerThread];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * THREADS;
    v[k] = 0.f;
    if (i < hidden) {
      float s = f32(xr[i]);
      if (ar) {
        s = round_to<T>(s + f32(ar[i]));
        xr[i] = Elem<T>::from_float(s);
      }
      v[k] = s;
      ss = fmaf(s, s, ss);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < THREADS / 32; ++k) tot += red[k];
  const float r = rsqrtf(tot / (float)hidden + eps);
  T* orow = out + row * o_st;
#pragma unroll
  for (int k = 0; k < kMaxPerThread; ++k) {
    const int i = threadIdx.x + k * THREADS;
    if (i < hidden) orow[i] = Elem<T>::from_float(v[k] * r * f32(w[i]));
  }
}

// out[t, f] = silu(gu[t, f]) * gu[t, ffn + f], fp32 inside, one rounding.
template <typename T>
__global__ void __launch_bounds__(256) swiglu_kernel(const T* gu, int64_t gu_st, T* out, int64_t o_st, int64_t n_rows,
                                                     int ffn) {
  const int64_t total = n_rows * (int64_t)ffn;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = e / ffn;
    const int f = (int)(e - row * ffn);
    const float g = f32(gu[row * gu_st + f]);
    const float u = f32(gu[row * gu_st + ffn + f]);
    out[row * o_st + f] = Elem<T>::from_float(g / (1.f + __expf(-g)) * u);
  }
}

// add_rmsnorm_kernel with 16-byte accesses: hidden % 8 == 0 and every row
// 16-byte aligned; a thread holds up to kMaxVec vectors of its row.
template <typename T, int THREADS>
__global__ void __launch_bounds__(THREADS) add_rmsnorm_vec_kernel(T* x, int64_t x_st, const T* a, int64_t a_st,
                                                                  const T* w, T* out, int64_t o_st, int hidden,
                                                                  float eps) {
  constexpr int kMaxVec = 4;
  __shared__ float red[THREADS / 32];
  const int64_t row = blockIdx.x;
  const int nvec = hidden / 8;
  uint4* xr = reinterpret_cast<uint4*>(x + row * x_st);
  const uint4* ar = a ? reinterpret_cast<const uint4*>(a + row * a_st) : nullptr;
  Vec8<T> v[kMaxVec];
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * THREADS;
    if (i < nvec) {
      v[k].raw = xr[i];
      if (ar) {
        Vec8<T> r;
        r.raw = ar[i];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[k].set(e, v[k].get(e) + r.get(e));  // rounded to T, like the eager add
        xr[i] = v[k].raw;
      }
    }
  }
  const float r = rms_scale<T, THREADS, kMaxVec>(v, nvec, hidden, eps, red);
  uint4* orow = reinterpret_cast<uint4*>(out + row * o_st);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int k = 0; k < kMaxVec; ++k) {
    const int i = threadIdx.x + k * THREADS;
    if (i < nvec) {
      Vec8<T> wk, o;
      wk.raw = __ldg(wv + i);
#pragma unroll
      for (int e = 0; e < 8; ++e) o.set(e, v[k].get(e) * r * wk.get(e));
      orow[i] = o.raw;
    }
  }
}

// swiglu_kernel with 16-byte accesses: ffn % 8 == 0, rows 16-byte aligned; grid
// (vector blocks, rows).
template <typename T>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(const T* gu, int64_t gu_st, T* out, int64_t o_st, int ffn) {
  const int64_t row = blockIdx.y;
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= ffn / 8) return;
  const uint4* g4 = reinterpret_cast<const uint4*>(gu + row * gu_st);
  Vec8<T> g, u, o;
  g.raw = __ldg(g4 + i);
  u.raw = __ldg(g4 + ffn / 8 + i);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float gv = g.get(e);
    o.set(e, gv / (1.f + __expf(-gv)) * u.get(e));
  }
  reinterpret_cast<uint4*>(out + row * o_st)[i] = o.raw;
}

template <typename T, int THREADS>
void launch_norm(T* x, int64_t x_st, const T* a, int64_t a_st, const T* w, T* out, int64_t o_st, int64_t n, int hidden,
                 float eps, cudaStream_t s) {
  add_rmsnorm_kernel<T, THREADS><<<(unsigned)n, THREADS, 0, s>>>(x, x_st, a, a_st, w, out, o_st, hidden, eps);
}

}  // namespace
}  // namespace seb

extern "C" int seb_rope_kv_append(const void* qkv, int64_t qkv_stride_token, int64_t n_tokens, int32_t num_q_heads,
                                  int32_t num_kv_heads, int32_t head_dim, const void* cos, const void* sin,
                                  int64_t cos_sin_stride_token, const int64_t* slot_mapping, void* q_out,
                                  int64_t q_out_stride_token, void* k_cache, void* v_cache, int64_t num_blocks,
                                  int32_t dtype, int32_t* err, void* stream) {
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(dtype == SEB_BF16 || dtype == SEB_F16, "seb_rope_kv_append: bf16 or fp16 required (dtype %d)", dtype);
  SEB_CHECK_ARG(n_tokens >= 0, "seb_rope_kv_append: n_tokens < 0");
  SEB_CHECK_ARG(num_q_heads > 0 && num_kv_heads > 0 && head_dim > 0 && head_dim % 2 == 0 && num_blocks > 0,
                "seb_rope_kv_append: head counts, an even head_dim and num_blocks must be positive");
  if (n_tokens == 0) return SEB_OK;
  SEB_CHECK_ARG(qkv && cos && sin && slot_mapping && q_out && k_cache && v_cache,
                "seb_rope_kv_append: NULL pointer argument");
  SEB_CHECK_ARG(qkv_stride_token >= (int64_t)(num_q_heads + 2 * num_kv_heads) * head_dim &&
                    q_out_stride_token >= (int64_t)num_q_heads * head_dim && cos_sin_stride_token >= head_dim,
                "seb_rope_kv_append: a token stride is smaller than its row");
  RopeParams p;
  p.qkv = static_cast<const char*>(qkv);
  p.qkv_st = qkv_stride_token * 2;
  p.cos = static_cast<const char*>(cos);
  p.sin = static_cast<const char*>(sin);
  p.cs_st = cos_sin_stride_token * 2;
  p.slots = slot_mapping;
  p.num_slots = num_blocks * kBlockSize;
  p.q_out = static_cast<char*>(q_out);
  p.q_st = q_out_stride_token * 2;
  p.k_cache = static_cast<char*>(k_cache);
  p.v_cache = static_cast<char*>(v_cache);
  p.n_tokens = n_tokens;
  p.hq = num_q_heads;
  p.hkv = num_kv_heads;
  p.d = head_dim;
  p.err = err;
  p.pairs = head_dim % 4 == 0 && aligned(qkv, 4) && aligned(cos, 4) && aligned(sin, 4) && aligned(q_out, 4) &&
            aligned(k_cache, 4) && aligned(v_cache, 4) && qkv_stride_token % 2 == 0 && cos_sin_stride_token % 2 == 0 &&
            q_out_stride_token % 2 == 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec16 = head_dim % 16 == 0 && aligned(qkv, 16) && aligned(cos, 16) && aligned(sin, 16) &&
                     aligned(q_out, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) &&
                     qkv_stride_token % 8 == 0 && cos_sin_stride_token % 8 == 0 && q_out_stride_token % 8 == 0;
  if (vec16) {
    const int64_t threads = n_tokens * (int64_t)(num_q_heads + 3 * num_kv_heads) * (head_dim / 16);
    const int64_t blocks = (threads + 255) / 256;
    SEB_CHECK_ARG(blocks < (1ll << 31), "seb_rope_kv_append: too many tokens");
    if (dtype == SEB_BF16)
      rope_append_vec_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(p);
    else
      rope_append_vec_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(p);
    return launch_status("rope_append_vec_kernel");
  }
  const int64_t warps = n_tokens * (num_q_heads + 2 * num_kv_heads);
  const int64_t blocks = (warps + 7) / 8;
  SEB_CHECK_ARG(blocks < (1ll << 31), "seb_rope_kv_append: too many tokens");
  if (dtype == SEB_BF16)
    rope_append_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(p);
  else
    rope_append_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(p);
  return launch_status("rope_append_kernel");
}

extern "C" int seb_add_rmsnorm(void* x, int64_t x_stride, const void* residual, int64_t residual_stride,
                               const void* weight, void* out, int64_t out_stride, int64_t n_rows, int32_t hidden,
                               float eps, int32_t dtype, void* stream) {
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(dtype == SEB_BF16 || dtype == SEB_F16, "seb_add_rmsnorm: bf16 or fp16 required (dtype %d)", dtype);
  SEB_CHECK_ARG(n_rows >= 0 && hidden > 0, "seb_add_rmsnorm: bad shape");
  SEB_CHECK_ARG(hidden <= 32 * 1024, "seb_add_rmsnorm: hidden %d above 32768", hidden);
  if (n_rows == 0) return SEB_OK;
  SEB_CHECK_ARG(x && weight && out, "seb_add_rmsnorm: NULL pointer argument");
  SEB_CHECK_ARG(n_rows < (1ll << 31), "seb_add_rmsnorm: too many rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = hidden % 8 == 0 && hidden <= 4 * 8 * 1024 && aligned(x, 16) && aligned(weight, 16) &&
                   aligned(out, 16) && (residual == nullptr || aligned(residual, 16)) && x_stride % 8 == 0 &&
                   out_stride % 8 == 0 && (residual == nullptr || residual_stride % 8 == 0);
  if (vec) {
    // up to 4 vectors of 8 per thread: 256 threads up to 8192, 1024 threads above
    const unsigned grid = (unsigned)n_rows;
    if (dtype == SEB_BF16) {
      using T = __nv_bfloat16;
      if (hidden <= 8192)
        add_rmsnorm_vec_kernel<T, 256><<<grid, 256, 0, s>>>(static_cast<T*>(x), x_stride, static_cast<const T*>(residual),
                                                           residual_stride, static_cast<const T*>(weight),
                                                           static_cast<T*>(out), out_stride, hidden, eps);
      else
        add_rmsnorm_vec_kernel<T, 1024><<<grid, 1024, 0, s>>>(static_cast<T*>(x), x_stride,
                                                             static_cast<const T*>(residual), residual_stride,
                                                             static_cast<const T*>(weight), static_cast<T*>(out),
                                                             out_stride, hidden, eps);
    } else {
      using T = __half;
      if (hidden <= 8192)
        add_rmsnorm_vec_kernel<T, 256><<<grid, 256, 0, s>>>(static_cast<T*>(x), x_stride, static_cast<const T*>(residual),
                                                           residual_stride, static_cast<const T*>(weight),
                                                           static_cast<T*>(out), out_stride, hidden, eps);
      else
        add_rmsnorm_vec_kernel<T, 1024><<<grid, 1024, 0, s>>>(static_cast<T*>(x), x_stride,
                                                             static_cast<const T*>(residual), residual_stride,
                                                             static_cast<const T*>(weight), static_cast<T*>(out),
                                                             out_stride, hidden, eps);
    }
    return launch_status("add_rmsnorm_vec_kernel");
  }
  // 32 values per thread at most: 256 threads up to 8192, 1024 threads above.
  if (dtype == SEB_BF16) {
    using T = __nv_bfloat16;
    if (hidden <= 8192)
      launch_norm<T, 256>(static_cast<T*>(x), x_stride, static_cast<const T*>(residual), residual_stride,
                          static_cast<const T*>(weight), static_cast<T*>(out), out_stride, n_rows, hidden, eps, s);
    else
      launch_norm<T, 1024>(static_cast<T*>(x), x_stride, static_cast<const T*>(residual), residual_stride,
                           static_cast<const T*>(weight), static_cast<T*>(out), out_stride, n_rows, hidden, eps, s);
  } else {
    using T = __half;
    if (hidden <= 8192)
      launch_norm<T, 256>(static_cast<T*>(x), x_stride, static_cast<const T*>(residual), residual_stride,
                          static_cast<const T*>(weight), static_cast<T*>(out), out_stride, n_rows, hidden, eps, s);
    else
      launch_norm<T, 1024>(static_cast<T*>(x), x_stride, static_cast<const T*>(residual), residual_stride,
                           static_cast<const T*>(weight), static_cast<T*>(out), out_stride, n_rows, hidden, eps, s);
  }
  return launch_status("add_rmsnorm_kernel");
}

extern "C" int seb_swiglu(const void* gate_up, int64_t gate_up_stride, void* out, int64_t out_stride, int64_t n_rows,
                          int32_t ffn, int32_t dtype, void* stream) {
  using namespace seb;
  clear_error();
  SEB_CHECK_ARG(dtype == SEB_BF16 || dtype == SEB_F16, "seb_swiglu: bf16 or fp16 required (dtype %d)", dtype);
  SEB_CHECK_ARG(n_rows >= 0 && ffn > 0, "seb_swiglu: bad shape");
  if (n_rows == 0) return SEB_OK;
  SEB_CHECK_ARG(gate_up && out, "seb_swiglu: NULL pointer argument");
  SEB_CHECK_ARG(gate_up_stride >= 2 * (int64_t)ffn && out_stride >= ffn, "seb_swiglu: a row stride is too small");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (ffn % 8 == 0 && aligned(gate_up, 16) && aligned(out, 16) && gate_up_stride % 8 == 0 && out_stride % 8 == 0 &&
      n_rows <= 65535) {
    const dim3 grid((unsigned)((ffn / 8 + 255) / 256), (unsigned)n_rows);
    if (dtype == SEB_BF16)
      swiglu_vec_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gate_up),
                                                             gate_up_stride, static_cast<__nv_bfloat16*>(out),
                                                             out_stride, ffn);
    else
      swiglu_vec_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(gate_up), gate_up_stride,
                                                      static_cast<__half*>(out), out_stride, ffn);
    return launch_status("swiglu_vec_kernel");
  }
  const int64_t total = n_rows * (int64_t)ffn;
  const int64_t blocks = std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 16);
  if (dtype == SEB_BF16)
    swiglu_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, s>>>(
        static_cast<const __nv_bfloat16*>(gate_up), gate_up_stride, static_cast<__nv_bfloat16*>(out), out_stride,
        n_rows, ffn);
  else
    swiglu_kernel<__half><<<(unsigned)blocks, 256, 0, s>>>(static_cast<const __half*>(gate_up), gate_up_stride,
                                                           static_cast<__half*>(out), out_stride, n_rows, ffn);
  return launch_status("swiglu_kernel");
}
