// CPU oracle for the PagedAttention decode path — TEST INFRASTRUCTURE ONLY.
//
// Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
// arm may load this library, and only as the checker or the timed CPU
// baseline; the product path (libclove_cuda.so) never calls it.
//
// PARITY UNPINNED.  The reference (rakeshpdey/clove, Rust) cannot be built or
// run here (no Rust toolchain; its only PagedAttention kernel is WGSL run
// through wgpu, which needs a graphics stack that is unavailable on this box),
// its eager CPU path panics (src/backend.rs:2937-2948), and its tests hold no
// PagedAttention vectors.  This file restates the semantics the reference
// documents for the op:
//   - softmax(q K^T * scale) V with the scale applied to q:
//       src/nn/attention.rs:52-69 (scale = 1/sqrt(head_dim) at :64)
//   - block-table gather: token t of sequence b lives in physical block
//       block_tables[b][t / block_size] at offset t % block_size:
//       src/lazy.rs:5259-5270 (there with a fixed table stride of 1024 and no
//       head index; here with an explicit stride and KV-head index)
//   - cache layout [num_blocks, block_size, num_heads, head_dim]:
//       src/nn.rs:534-536
//   - f32 arithmetic idiom of the reference CPU ops: a sequential f32 dot
//       product per output (rayon_matmul, src/backend.rs:266-287) and a row
//       softmax as max, exp(x - max), sum, divide (src/backend.rs:2107-2124),
//       run in parallel over independent rows as Rayon does.
//   - the literal placeholder kernel, for characterisation only:
//       src/lazy.rs:5255-5274.
// The KV append (absent in the reference) follows the slot rule
//   slot_b = block_tables[b][ctx_b / block_size] * block_size + ctx_b % block_size
// and decode then attends over ctx_b + 1 tokens.
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr int kF32 = 0, kF16 = 16, kBF16 = 160;

// Exact widening of the stored element to double/float.
inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline float f16_to_f32(uint16_t h) {
  // IEEE half -> single, written out (subnormals, inf, nan included).
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else {  // subnormal: normalise
      int e = -1;
      do {
        ++e;
        man <<= 1;
      } while ((man & 0x400u) == 0);
      man &= 0x3ffu;
      u = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (man << 13);
  } else {
    u = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline float load_elem(const void* base, size_t i, int dtype) {
  if (dtype == kF32) return static_cast<const float*>(base)[i];
  uint16_t h = static_cast<const uint16_t*>(base)[i];
  return dtype == kBF16 ? bf16_to_f32(h) : f16_to_f32(h);
}

struct Geom {
  int dtype, batch, hq, hkv, d, bs, bt_stride, num_blocks;
  const void* q;
  const void* kc;
  const void* vc;
  const int32_t* bt;
  const int32_t* ctx;
};

// Row offset (in elements) of token t, KV head h of sequence b; -1 if the
// block-table entry is out of range.
inline long long row_of(const Geom& g, int b, int t, int h) {
  int phys = g.bt[(size_t)b * g.bt_stride + t / g.bs];
  if (phys < 0 || phys >= g.num_blocks) return -1;
  return (((long long)phys * g.bs + t % g.bs) * g.hkv + h) * g.d;
}

template <typename F>
void parallel_for(int n, int nthreads, F&& f) {
  if (nthreads <= 1 || n <= 1) {
    for (int i = 0; i < n; ++i) f(i);
    return;
  }
  std::vector<std::thread> pool;
  std::atomic_int next{0};
  for (int t = 0; t < nthreads; ++t) {
    pool.emplace_back([&] {
      for (int i = next.fetch_add(1); i < n; i = next.fetch_add(1)) f(i);
    });
  }
  for (auto& th : pool) th.join();
}

}  // namespace

extern "C" {

// Bit-exact KV append: copy row i of k/v (row_bytes each) to slot
// slot_mapping[i]; negative slots are padding and skipped.  Returns the
// number of slots that were out of range (and skipped).
int oracle_reshape_and_cache(void* k_cache, void* v_cache, const void* k, const void* v, const int32_t* slots,
                             int num_tokens, int row_bytes, long long num_slots) {
  int bad = 0;
  for (int i = 0; i < num_tokens; ++i) {
    int s = slots[i];
    if (s < 0) continue;
    if (s >= num_slots) {
      ++bad;
      continue;
    }
    std::memcpy(static_cast<char*>(k_cache) + (size_t)s * row_bytes, static_cast<const char*>(k) + (size_t)i * row_bytes,
                row_bytes);
    std::memcpy(static_cast<char*>(v_cache) + (size_t)s * row_bytes, static_cast<const char*>(v) + (size_t)i * row_bytes,
                row_bytes);
  }
  return bad;
}

// Slot of each sequence's appended token (ctx_b is the pre-append length).
void oracle_append_slots(const int32_t* bt, int bt_stride, const int32_t* ctx, int batch, int block_size,
                         int32_t* slots) {
  for (int b = 0; b < batch; ++b) {
    int c = ctx[b];
    slots[b] = bt[(size_t)b * bt_stride + c / block_size] * block_size + c % block_size;
  }
}

// Bit-exact gather to [batch, max_ctx, row] (row = num_kv_heads*head_dim
// elements, row_bytes bytes), zero rows past each context length.  Returns
// the number of out-of-range block-table entries met.
int oracle_gather_kv(const void* k_cache, const void* v_cache, const int32_t* bt, int bt_stride, const int32_t* ctx,
                     int batch, int max_ctx, int block_size, int num_blocks, int row_bytes, void* k_out,
                     void* v_out) {
  int bad = 0;
  for (int b = 0; b < batch; ++b) {
    int c = ctx[b];
    if (c < 0) c = 0;
    if (c > max_ctx) c = max_ctx;
    if (c > bt_stride * block_size) c = bt_stride * block_size;
    for (int t = 0; t < max_ctx; ++t) {
      char* ko = static_cast<char*>(k_out) + ((size_t)b * max_ctx + t) * row_bytes;
      char* vo = static_cast<char*>(v_out) + ((size_t)b * max_ctx + t) * row_bytes;
      int phys = t < c ? bt[(size_t)b * bt_stride + t / block_size] : -1;
      if (t < c && (phys < 0 || phys >= num_blocks)) ++bad;
      if (t >= c || phys < 0 || phys >= num_blocks) {
        std::memset(ko, 0, row_bytes);
        std::memset(vo, 0, row_bytes);
        continue;
      }
      size_t src = ((size_t)phys * block_size + t % block_size) * row_bytes;
      std::memcpy(ko, static_cast<const char*>(k_cache) + src, row_bytes);
      std::memcpy(vo, static_cast<const char*>(v_cache) + src, row_bytes);
    }
  }
  return bad;
}

// fp64 ground truth.  q: [batch, hq, d]; out: double [batch, hq, d].  A
// sequence with context length 0 gets zeros.
void oracle_decode_f64(int dtype, const void* q, const void* k_cache, const void* v_cache, const int32_t* bt,
                       int bt_stride, const int32_t* ctx, int batch, int hq, int hkv, int d, int block_size,
                       int num_blocks, double scale, double* out, int nthreads) {
  Geom g{dtype, batch, hq, hkv, d, block_size, bt_stride, num_blocks, q, k_cache, v_cache, bt, ctx};
  const int grp = hq / hkv;
  parallel_for(batch * hq, nthreads, [&](int task) {
    const int b = task / hq, h = task % hq, kvh = h / grp;
    const int L = ctx[b];
    double* o = out + (size_t)task * d;
    for (int i = 0; i < d; ++i) o[i] = 0.0;
    if (L <= 0) return;
    std::vector<double> qs(d), s(L);
    for (int i = 0; i < d; ++i) qs[i] = (double)load_elem(q, (size_t)task * d + i, dtype) * scale;
    double mx = -INFINITY;
    for (int t = 0; t < L; ++t) {
      long long r = row_of(g, b, t, kvh);
      double acc = 0.0;
      if (r >= 0)
        for (int i = 0; i < d; ++i) acc += qs[i] * (double)load_elem(k_cache, (size_t)r + i, dtype);
      s[t] = acc;
      if (acc > mx) mx = acc;
    }
    double sum = 0.0;
    for (int t = 0; t < L; ++t) {
      s[t] = std::exp(s[t] - mx);
      sum += s[t];
    }
    for (int t = 0; t < L; ++t) {
      long long r = row_of(g, b, t, kvh);
      if (r < 0) continue;
      double p = s[t] / sum;
      for (int i = 0; i < d; ++i) o[i] += p * (double)load_elem(v_cache, (size_t)r + i, dtype);
    }
  });
}

// f32 restatement in the reference CPU ops' idiom (the timed CPU baseline).
// Parallel tasks are (sequence, KV head); each task handles the query heads
// of that KV head, computing in f32:
//   q_s = q * scale                          (src/nn/attention.rs:63-64)
//   s_t = sum_p q_s[p] * K_t[p]  sequential  (src/backend.rs:276-283)
//   P   = softmax(s): max, exp(s-max), sum, divide (src/backend.rs:2114-2123)
//   o_d = sum_t P_t * V_t[d]     sequential  (src/backend.rs:276-283)
void oracle_decode_f32(int dtype, const void* q, const void* k_cache, const void* v_cache, const int32_t* bt,
                       int bt_stride, const int32_t* ctx, int batch, int hq, int hkv, int d, int block_size,
                       int num_blocks, float scale, float* out, int nthreads) {
  Geom g{dtype, batch, hq, hkv, d, block_size, bt_stride, num_blocks, q, k_cache, v_cache, bt, ctx};
  const int grp = hq / hkv;
  parallel_for(batch * hkv, nthreads, [&](int task) {
    const int b = task / hkv, kvh = task % hkv;
    const int L = ctx[b];
    std::vector<float> qs(d), s(L > 0 ? L : 1), kt, vt;
    // Gather this (sequence, head)'s K and V rows as dense f32 [L, d], the
    // layout the reference matmul consumes.
    kt.assign((size_t)(L > 0 ? L : 0) * d, 0.f);
    vt.assign((size_t)(L > 0 ? L : 0) * d, 0.f);
    for (int t = 0; t < L; ++t) {
      long long r = row_of(g, b, t, kvh);
      if (r < 0) continue;
      for (int i = 0; i < d; ++i) {
        kt[(size_t)t * d + i] = load_elem(k_cache, (size_t)r + i, dtype);
        vt[(size_t)t * d + i] = load_elem(v_cache, (size_t)r + i, dtype);
      }
    }
    for (int gq = 0; gq < grp; ++gq) {
      const int h = kvh * grp + gq;
      float* o = out + ((size_t)b * hq + h) * d;
      if (L <= 0) {
        for (int i = 0; i < d; ++i) o[i] = 0.f;
        continue;
      }
      const size_t qoff = ((size_t)b * hq + h) * d;
      for (int i = 0; i < d; ++i) qs[i] = load_elem(q, qoff + i, dtype) * scale;
      for (int t = 0; t < L; ++t) {
        float sum = 0.f;
        const float* kr = &kt[(size_t)t * d];
        for (int p = 0; p < d; ++p) sum += qs[p] * kr[p];
        s[t] = sum;
      }
      float mx = -INFINITY;
      for (int t = 0; t < L; ++t) mx = s[t] > mx ? s[t] : mx;
      float tot = 0.f;
      for (int t = 0; t < L; ++t) {
        float e = std::exp(s[t] - mx);
        s[t] = e;
        tot += e;
      }
      for (int t = 0; t < L; ++t) s[t] /= tot;
      for (int i = 0; i < d; ++i) {
        float sum = 0.f;
        for (int t = 0; t < L; ++t) sum += s[t] * vt[(size_t)t * d + i];
        o[i] = sum;
      }
    }
  });
}

// Literal restatement of the reference's placeholder WGSL kernel
// (src/lazy.rs:5255-5274), for characterisation only: one output element per
// index i < size, out[i] = q[i] * kv_cache[phys*bs*hd + off*hd + i%hd] *
// (1/sqrt(hd)) with the fixed table stride of 1024.  Not the op's semantics.
void oracle_mock_paged_attention(const float* q, const float* kv_cache, const uint32_t* block_tables,
                                 unsigned size, unsigned seq_len, unsigned head_dim, unsigned block_size,
                                 float* out) {
  const float scale = 1.0f / std::sqrt((float)head_dim);
  for (unsigned i = 0; i < size; ++i) {
    unsigned token_idx = i % seq_len;
    unsigned logical = token_idx / block_size;
    unsigned off = token_idx % block_size;
    unsigned batch_idx = i / (seq_len * head_dim);
    unsigned phys = block_tables[batch_idx * 1024u + logical];
    float k_val = kv_cache[phys * block_size * head_dim + off * head_dim + (i % head_dim)];
    out[i] = q[i] * k_val * scale;
  }
}

}  // extern "C"
