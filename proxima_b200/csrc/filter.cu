// filter.cu — typed metadata filters evaluated on the device.
//
// The reference evaluates `MetadataFilter::accepts` (crates/proxima-server/src/
// filter.rs:216-256) once per candidate on the host; a batched search instead
// needs the accepted set as a bitmap over slots, and building it on the host
// costs a closure call per live slot per batch. Here the fields a filter
// reads are held as typed device columns (one type tag and one 64-bit payload
// per slot), the compiled conditions are evaluated by one thread per slot,
// and the bitmap every search entry point takes is written directly.
//
// Semantics, condition by condition (all must hold; filter.rs:216-256):
//   * an absent field fails every condition except exists:false;
//   * eq / ne compare MetadataValue as its derived PartialEq does: same variant
//     and equal payload (f64 ==, so NaN != NaN and -0.0 == 0.0);
//   * gt / gte / lt / lte take a numeric bound: Int bound vs Int field by
//     integer order, Float bound vs Float field by f64::total_cmp, Int bound vs
//     Float field by total_cmp against the bound as f64; any other pairing
//     fails (filter.rs:81-97);
//   * in holds when some operand equals the value;
//   * exists:b holds when the field's presence equals b.
#include <algorithm>
#include <new>
#include <vector>

#include "common.cuh"

namespace pxc {
namespace flt {

// f64::total_cmp as a signed integer key.
__device__ __forceinline__ int64_t total_key(int64_t bits) {
  return bits ^ (int64_t)(((uint64_t)(bits >> 63)) >> 1);
}

__device__ __forceinline__ bool value_eq(uint32_t ta, int64_t a, uint32_t tb, int64_t b) {
  if (ta != tb) return false;
  if (ta == PXC_VALUE_FLOAT) return __longlong_as_double(a) == __longlong_as_double(b);
  return a == b;
}

// Ordering of the field against a numeric bound: -1, 0, 1, or 2 when the
// pairing is not comparable (Number::compare, filter.rs:81-97).
__device__ __forceinline__ int compare_bound(uint32_t tb, int64_t bound, uint32_t tv, int64_t v) {
  if (tb == PXC_VALUE_INT && tv == PXC_VALUE_INT) return v < bound ? -1 : (v > bound ? 1 : 0);
  int64_t fb;
  if (tb == PXC_VALUE_FLOAT && tv == PXC_VALUE_FLOAT)
    fb = bound;
  else if (tb == PXC_VALUE_INT && tv == PXC_VALUE_FLOAT)
    fb = __double_as_longlong((double)bound);
  else
    return 2;
  const int64_t kv = total_key(v), kb = total_key(fb);
  return kv < kb ? -1 : (kv > kb ? 1 : 0);
}

struct DevColumn {
  const uint8_t* tags;
  const int64_t* values;
  uint64_t n;  // slots the column covers; later slots are absent
};

// One thread per slot; warps vote the bitmap's 32-bit halves.
__global__ void eval_kernel(const DevColumn* __restrict__ cols, uint32_t ncols, const pxc_condition* __restrict__ conds,
                            uint32_t ncond, const pxc_operand* __restrict__ ops, uint64_t nslots,
                            uint32_t* __restrict__ bitmap32) {
  const uint64_t s = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  bool ok = s < nslots;
  for (uint32_t c = 0; c < ncond && ok; ++c) {
    const pxc_condition cd = conds[c];
    uint32_t tv = PXC_VALUE_ABSENT;
    int64_t v = 0;
    if (cd.column < ncols && s < cols[cd.column].n) {
      tv = cols[cd.column].tags[s];
      v = cols[cd.column].values[s];
    }
    bool held;
    if (cd.op == PXC_COND_EXISTS) {
      held = (tv != PXC_VALUE_ABSENT) == (cd.value != 0);
    } else if (tv == PXC_VALUE_ABSENT) {
      held = false;
    } else {
      switch (cd.op) {
        case PXC_COND_EQ: held = value_eq(tv, v, cd.tag, cd.value); break;
        case PXC_COND_NE: held = !value_eq(tv, v, cd.tag, cd.value); break;
        case PXC_COND_GT: held = compare_bound(cd.tag, cd.value, tv, v) == 1; break;
        case PXC_COND_GE: {
          const int o = compare_bound(cd.tag, cd.value, tv, v);
          held = o == 1 || o == 0;
          break;
        }
        case PXC_COND_LT: held = compare_bound(cd.tag, cd.value, tv, v) == -1; break;
        case PXC_COND_LE: {
          const int o = compare_bound(cd.tag, cd.value, tv, v);
          held = o == -1 || o == 0;
          break;
        }
        case PXC_COND_IN: {
          held = false;
          const uint64_t first = (uint64_t)cd.value;
          for (uint32_t i = 0; i < cd.count && !held; ++i) held = value_eq(tv, v, ops[first + i].tag, ops[first + i].value);
          break;
        }
        default: held = false;
      }
    }
    ok = held;
  }
  const uint32_t vote = __ballot_sync(0xFFFFFFFFu, ok);
  const uint64_t base = s - (threadIdx.x & 31);
  if ((threadIdx.x & 31) == 0 && base < nslots) bitmap32[base / 32] = vote;
}

}  // namespace flt
}  // namespace pxc

using namespace pxc;

struct pxc_columns {
  pxc_ctx* ctx = nullptr;
  std::vector<DBuf<uint8_t>*> tags;
  std::vector<DBuf<int64_t>*> values;
  std::vector<uint64_t> len;  // slots written per column
  DBuf<flt::DevColumn> dcols;
  DBuf<pxc_condition> dconds;
  DBuf<pxc_operand> dops;
  std::mutex mu;
  ~pxc_columns() {
    for (auto* p : tags) delete p;
    for (auto* p : values) delete p;
  }
};

extern "C" {

pxc_status pxc_columns_create(pxc_ctx* ctx, pxc_columns** out, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(ctx != nullptr && out != nullptr, "ctx", 0, "null argument");
    pxc_columns* c = new (std::nothrow) pxc_columns();
    if (!c) throw make_failure(PXC_INTERNAL, 0, 0, nullptr, "out of host memory");
    c->ctx = ctx;
    *out = c;
  });
}

void pxc_columns_destroy(pxc_columns* c) {
  if (!c) return;
  int prev = -1;
  cudaGetDevice(&prev);
  cudaSetDevice(c->ctx->device);
  cudaStreamSynchronize(c->ctx->stream);
  delete c;
  if (prev >= 0) cudaSetDevice(prev);
}

pxc_status pxc_columns_set(pxc_columns* c, uint32_t column, const uint8_t* tags, const int64_t* values,
                           uint64_t slot_begin, uint64_t nslots, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(c != nullptr, "columns", 0, "null handle");
    PXC_CONFIG(column < 4096, "column", column, "at most 4096 columns");
    PXC_CONFIG(nslots == 0 || (tags != nullptr && values != nullptr), "tags", 0, "null buffer");
    for (uint64_t i = 0; i < nslots; ++i)
      if (tags[i] > PXC_VALUE_BOOL)
        throw make_failure(PXC_CONFIGURATION, tags[i], 0, "tags", "slot %llu has an unknown value tag",
                           (unsigned long long)(slot_begin + i));
    std::lock_guard<std::mutex> lock(c->mu);
    DeviceGuard g(c->ctx->device);
    cudaStream_t s = c->ctx->stream;
    while (c->tags.size() <= column) {
      c->tags.push_back(new DBuf<uint8_t>());
      c->values.push_back(new DBuf<int64_t>());
      c->len.push_back(0);
    }
    const uint64_t end = slot_begin + nslots;
    DBuf<uint8_t>& t = *c->tags[column];
    DBuf<int64_t>& v = *c->values[column];
    if (end > t.n) {
      const uint64_t cap = std::max<uint64_t>(end, t.n + t.n / 2);
      t.grow_keep(cap, c->len[column], s);
      v.grow_keep(cap, c->len[column], s);
    }
    if (slot_begin > c->len[column]) {  // a gap reads as absent
      PXC_CUDA(cudaMemsetAsync(t.p + c->len[column], 0, slot_begin - c->len[column], s));
      PXC_CUDA(cudaMemsetAsync(v.p + c->len[column], 0, (slot_begin - c->len[column]) * 8, s));
    }
    if (nslots) {
      PXC_CUDA(cudaMemcpyAsync(t.p + slot_begin, tags, nslots, cudaMemcpyHostToDevice, s));
      PXC_CUDA(cudaMemcpyAsync(v.p + slot_begin, values, nslots * 8, cudaMemcpyHostToDevice, s));
    }
    c->len[column] = std::max(c->len[column], end);
    PXC_CUDA(cudaStreamSynchronize(s));
  });
}

pxc_status pxc_columns_truncate(pxc_columns* c, uint64_t nslots, pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(c != nullptr, "columns", 0, "null handle");
    std::lock_guard<std::mutex> lock(c->mu);
    for (uint64_t& l : c->len) l = std::min(l, nslots);
  });
}

pxc_status pxc_columns_eval(pxc_columns* c, uint64_t nslots, const pxc_condition* conds, uint32_t ncond,
                            const pxc_operand* operands, uint32_t noperands, uint64_t* d_bitmap, void* stream,
                            pxc_error* err) {
  return guarded(err, [&] {
    PXC_CONFIG(c != nullptr, "columns", 0, "null handle");
    PXC_CONFIG(ncond == 0 || conds != nullptr, "conditions", 0, "null conditions");
    PXC_CONFIG(noperands == 0 || operands != nullptr, "operands", 0, "null operands");
    for (uint32_t i = 0; i < ncond; ++i) {
      const pxc_condition& cd = conds[i];
      PXC_CONFIG(cd.op <= PXC_COND_EXISTS, "op", cd.op, "unknown condition operator");
      if (cd.op == PXC_COND_IN)
        PXC_CONFIG(cd.value >= 0 && (uint64_t)cd.value + cd.count <= noperands && cd.count > 0, "in", cd.count,
                   "an 'in' list must be non-empty and lie inside the operands");
      if (cd.op >= PXC_COND_GT && cd.op <= PXC_COND_LE)
        PXC_CONFIG(cd.tag == PXC_VALUE_INT || cd.tag == PXC_VALUE_FLOAT, "bound", cd.tag,
                   "a range condition needs a numeric bound");
    }
    if (nslots == 0) return;
    PXC_CONFIG(d_bitmap != nullptr, "bitmap", 0, "null bitmap");
    std::lock_guard<std::mutex> lock(c->mu);
    DeviceGuard g(c->ctx->device);
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->ctx->stream;
    std::vector<flt::DevColumn> cols(c->tags.size());
    for (size_t i = 0; i < cols.size(); ++i) cols[i] = {c->tags[i]->p, c->values[i]->p, c->len[i]};
    c->dcols.reserve(std::max<size_t>(1, cols.size()));
    c->dconds.reserve(std::max<uint32_t>(1, ncond));
    c->dops.reserve(std::max<uint32_t>(1, noperands));
    if (!cols.empty())
      PXC_CUDA(cudaMemcpyAsync(c->dcols.p, cols.data(), cols.size() * sizeof(flt::DevColumn), cudaMemcpyHostToDevice, s));
    if (ncond) PXC_CUDA(cudaMemcpyAsync(c->dconds.p, conds, ncond * sizeof(pxc_condition), cudaMemcpyHostToDevice, s));
    if (noperands)
      PXC_CUDA(cudaMemcpyAsync(c->dops.p, operands, noperands * sizeof(pxc_operand), cudaMemcpyHostToDevice, s));
    // the last word's unused high bits stay zero
    const uint64_t words = (nslots + 63) / 64;
    PXC_CUDA(cudaMemsetAsync(d_bitmap, 0, words * 8, s));
    flt::eval_kernel<<<(unsigned)((nslots + 255) / 256), 256, 0, s>>>(c->dcols.p, (uint32_t)cols.size(), c->dconds.p,
                                                                      ncond, c->dops.p, nslots,
                                                                      reinterpret_cast<uint32_t*>(d_bitmap));
    PXC_CUDA(cudaGetLastError());
    c->ctx->launches += 1;
    PXC_CUDA(cudaStreamSynchronize(s));  // the condition copies are reused by the next call
  });
}

}  // extern "C"
