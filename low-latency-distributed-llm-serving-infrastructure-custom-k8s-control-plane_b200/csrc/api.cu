// C ABI of libb200paged.so (include/b200_paged.h): argument validation, plans, tensor maps and
// kernel launches.  No torch types; every entry point works on raw device pointers and a stream.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "attention.cuh"
#include "cache_ops.cuh"
#include "nvtx.cuh"

namespace {

thread_local std::string g_last_error;

int cuda_fail(cudaError_t e, const char* where) {
  g_last_error = std::string(where) + ": " + cudaGetErrorString(e);
  return B200_ERR_CUDA;
}

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int esize_of(int dtype) {
  switch (dtype) {
    case B200_DTYPE_F32: return 4;
    case B200_DTYPE_BF16: return 2;
    case B200_DTYPE_F16: return 2;
    default: return 0;
  }
}

// SM count of the calling thread's current device, cached per device (calls may come from
// several threads and devices).
int num_sms() {
  constexpr int kMaxDevices = 64;
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>* slot = (dev >= 0 && dev < kMaxDevices) ? &cache[dev] : nullptr;
  int n = slot ? slot->load(std::memory_order_relaxed) : 0;
  if (n == 0) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    if (slot) slot->store(n, std::memory_order_relaxed);
  }
  return n;
}

// ---- tensor maps -----------------------------------------------------------------------------
// cuTensorMapEncodeTiled is fetched through the runtime's driver entry point, so the library
// needs no link-time dependency on libcuda.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

struct MapKey {
  const void* ptr;
  int64_t rows;
  int32_t chunks, box_rows, dtype, row_bytes;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && chunks == o.chunks && box_rows == o.box_rows &&
           dtype == o.dtype && row_bytes == o.row_bytes;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ (std::hash<int64_t>()(k.rows) * 31) ^
           (static_cast<size_t>(k.chunks) << 20) ^ (static_cast<size_t>(k.box_rows) << 8);
  }
};

// A paged cache (L, NB, BS, Hkv, D) of 2-byte elements viewed as a 3-D tensor:
// dim0 = 64 elements (one 128-byte chunk of a head row), dim1 = Hkv * D/64 chunks of a token row,
// dim2 = L*NB*BS token rows.  Box = (64, 1, box_rows), 128-byte swizzle.
int cache_tensor_map(const void* cache, const B200CacheGeometry& g, int box_rows,
                     CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache_maps;
  const int64_t rows = static_cast<int64_t>(g.num_layers) * g.total_blocks * g.block_size;
  const int chunks = g.num_kv_heads * (g.head_dim / 64);
  const int row_bytes = g.num_kv_heads * g.head_dim * 2;
  MapKey key{cache, rows, chunks, box_rows, g.dtype, row_bytes};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache_maps.find(key);
  if (it != cache_maps.end()) {
    *out = it->second;
    return B200_OK;
  }
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(cache) % 16 != 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "cache pointer must be 16-byte aligned");
  CUtensorMap m;
  const cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(chunks), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = g.dtype == B200_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                            : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(&m, dt, 3, const_cast<void*>(cache), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  if (cache_maps.size() > 256) cache_maps.clear();
  cache_maps.emplace(key, m);
  *out = m;
  return B200_OK;
}

// Process-wide tuning knobs (b200_set_decode_split_tokens, b200_set_prefill_cuda_cores).
std::atomic<int> g_split_override{0};
std::atomic<bool> g_force_cuda_core_prefill{false};
std::atomic<int> g_prefill_kernel{1};
std::atomic<int> g_prefill_poly_exp{1};

struct DecodePlan {
  bool tensor_cores;
  int split_tokens;
  int nchunks, hpc, items_per_split;
  int64_t max_splits;
  size_t off_cu, off_work, off_cnt, off_lse, off_o, total;
};

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

int validate_geom(const B200CacheGeometry& g, int32_t layer_idx, int32_t hq) {
  if (esize_of(g.dtype) == 0) return fail(B200_ERR_UNSUPPORTED, "unsupported dtype");
  if (g.num_layers <= 0 || g.total_blocks <= 0 || g.block_size <= 0 || g.num_kv_heads <= 0 ||
      g.head_dim <= 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "cache geometry must be positive");
  if (hq <= 0 || hq % g.num_kv_heads != 0)
    return fail(B200_ERR_INVALID_ARGUMENT,
                "num_query_heads must be a multiple of num_kv_heads for GQA");
  if (layer_idx < 0 || layer_idx >= g.num_layers)
    return fail(B200_ERR_INVALID_ARGUMENT, "layer_idx out of range");
  if (g.head_dim > 256) return fail(B200_ERR_UNSUPPORTED, "head_dim > 256");
  return B200_OK;
}

bool tc_eligible(const B200CacheGeometry& g, const void* q, int64_t qs_row, int64_t qs_head,
                 const void* kc, const void* vc) {
  if (g.dtype != B200_DTYPE_BF16 && g.dtype != B200_DTYPE_F16) return false;
  if (g.head_dim != 64 && g.head_dim != 128) return false;
  if (!(g.block_size == 8 || g.block_size % 16 == 0)) return false;
  if (reinterpret_cast<uintptr_t>(q) % 4 != 0 || (qs_row & 1) || (qs_head & 1)) return false;
  if (reinterpret_cast<uintptr_t>(kc) % 16 != 0 || reinterpret_cast<uintptr_t>(vc) % 16 != 0)
    return false;
  const int64_t rows = static_cast<int64_t>(g.num_layers) * g.total_blocks * g.block_size;
  if (rows >= (int64_t(1) << 31)) return false;
  return true;
}

DecodePlan make_decode_plan(const B200DecodeParams& p) {
  DecodePlan pl{};
  const int G = p.num_query_heads / p.geom.num_kv_heads;
  pl.tensor_cores = tc_eligible(p.geom, p.query, p.q_stride_row, p.q_stride_head, p.key_cache,
                                p.value_cache);
  pl.nchunks = (G + 7) / 8;
  pl.hpc = G < 8 ? G : 8;
  pl.items_per_split = p.geom.num_kv_heads * pl.nchunks;
  const int64_t max_ctx = p.max_context_len > 0 ? p.max_context_len : 1;
  // Split size: 2048 tokens.  Each split writes and re-reads a partial and adds a merge, so
  // shorter splits only pay when a batch would otherwise leave most SMs without work: the split
  // halves (not below 512) while there are fewer (sequence, split, head) items than half the SMs.
  // Measured GB/s (bf16, GQA 4, D 128) for splits 512 / 1024 / 2048 / 4096: config 2 (256
  // sequences, lognormal <= 4096) 4666 / 5300 / 5549 / 5270; config 5 at TP 1 (14 sequences,
  // 8k-32k) 4476 / 4900 / 5207 / 5196; at TP 8 (115 sequences, one KV head) 4438 / 5063 / 5193 /
  // 5224; 64 sequences of ~600 tokens 2949 / 3195 / 3254 / 3250; 32 sequences <= 4096 2869 /
  // 2968 / 2872 / 2142; one 32k sequence 1702 / 2299 / 2479 / 1842.  (The earlier rule, at least
  // 16 items per SM, picked 1024 down to 64 on all but config 2: 339 GB/s for the 32k sequence.)
  int split = g_split_override.load(std::memory_order_relaxed);
  if (split <= 0) {
    split = 2048;
    while (split > 512 &&
           static_cast<int64_t>(p.num_seqs) * ((max_ctx + split - 1) / split) * pl.items_per_split <
               num_sms() / 2)
      split /= 2;
  }
  pl.split_tokens = split;
  pl.max_splits = static_cast<int64_t>(p.num_seqs) * ((max_ctx + split - 1) / split);
  size_t off = align256(sizeof(b200::DecodeHeader));
  pl.off_cu = off;
  off += align256((p.num_seqs + 1) * sizeof(int32_t));
  pl.off_work = off;
  off += align256(pl.max_splits * sizeof(int2));
  pl.off_cnt = off;
  off += align256(static_cast<size_t>(p.num_seqs) * pl.items_per_split * sizeof(int32_t));
  pl.off_lse = off;
  off += align256(static_cast<size_t>(pl.max_splits) * pl.items_per_split * pl.hpc * 4);
  pl.off_o = off;
  off += align256(static_cast<size_t>(pl.max_splits) * pl.items_per_split * pl.hpc *
                  p.geom.head_dim * 4);
  pl.total = pl.tensor_cores ? off : 0;
  return pl;
}

}  // namespace

namespace b200 {
void set_last_error(const char* msg) { g_last_error = msg; }
}  // namespace b200

extern "C" {

const char* b200_status_string(int status) {
  switch (status) {
    case B200_OK: return "ok";
    case B200_ERR_INVALID_ARGUMENT: return "invalid argument";
    case B200_ERR_OUT_OF_MEMORY: return "out of memory";
    case B200_ERR_OUT_OF_RANGE: return "out of range";
    case B200_ERR_RUNTIME: return "runtime error";
    case B200_ERR_UNSUPPORTED: return "unsupported";
    case B200_ERR_CUDA: return "cuda error";
    default: return "unknown status";
  }
}

const char* b200_last_error(void) { return g_last_error.c_str(); }

void b200_set_decode_split_tokens(int32_t tokens) {
  g_split_override.store(tokens > 0 ? ((tokens + 15) / 16) * 16 : 0, std::memory_order_relaxed);
}

// ---- reference-signature masked attention ---------------------------------------------------

int b200_paged_attention(const float* query, const float* key_cache, const float* value_cache,
                         int32_t layer_idx, PagedAttentionDims dims, const int32_t* gather_slots,
                         const uint8_t* attention_mask, float scaling, float* output,
                         int32_t* status_word, void* stream) {
  b200::NvtxRange nvtx_range("b200_paged_attention");
  B200CacheGeometry g{dims.num_layers, dims.total_blocks, dims.block_size, dims.num_kv_heads,
                      dims.head_dim, B200_DTYPE_F32};
  int rc = validate_geom(g, layer_idx, dims.num_query_heads);
  if (rc != B200_OK) return rc;
  if (dims.num_query_tokens < 0 || dims.num_context_tokens < 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "negative token counts");
  if (dims.num_query_tokens == 0) return B200_OK;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = dims.num_query_heads / dims.num_kv_heads;
  b200::RowArgs a{};
  a.mode = b200::kRowMask;
  a.q = query;
  a.q_srow = dims.head_dim;
  a.q_shead = static_cast<int64_t>(dims.num_query_tokens) * dims.head_dim;
  a.kc = key_cache;
  a.vc = value_cache;
  a.layer = layer_idx;
  a.nb = dims.total_blocks;
  a.bs = dims.block_size;
  a.hkv = dims.num_kv_heads;
  a.head_dim = dims.head_dim;
  a.group = G;
  a.nchunks = (G + 7) / 8;
  a.gather = gather_slots;
  a.mask = attention_mask;
  a.num_ctx = dims.num_context_tokens;
  a.scale = scaling;
  a.out = output;
  a.o_srow = static_cast<int64_t>(dims.num_query_heads) * dims.head_dim;
  a.o_shead = dims.head_dim;
  a.status = status_word;
  cudaError_t e = b200::launch_row(B200_DTYPE_F32, a, dims.num_query_tokens, st);
  if (e != cudaSuccess) return cuda_fail(e, "paged_attention");
  return B200_OK;
}

void paged_attention(const float* query, const float* key_cache, const float* value_cache,
                     const int32_t layer_idx, const PagedAttentionDims dims,
                     const int32_t* gather_slots, const uint8_t* attention_mask,
                     const float scaling, float* output, float* scratch, void* stream) {
  (void)scratch;
  b200_paged_attention(query, key_cache, value_cache, layer_idx, dims, gather_slots,
                       attention_mask, scaling, output, nullptr, stream);
}

// ---- decode ---------------------------------------------------------------------------------

size_t b200_paged_decode_workspace_bytes(const B200DecodeParams* p) {
  if (p == nullptr || p->num_seqs <= 0 || p->geom.num_kv_heads <= 0 ||
      p->num_query_heads % p->geom.num_kv_heads != 0)
    return 0;
  return make_decode_plan(*p).total;
}

}  // extern "C"

namespace {
// Decode over block tables.  cu_q != NULL: mixed batch, only sequences with exactly one new
// token (row cu_q[s]) are attended; the others are left to the prefill kernel.
int run_decode(const B200DecodeParams& p, const int64_t* cu_q, void* workspace,
               size_t workspace_bytes, cudaStream_t st) {
  int rc = B200_OK;
  const int G = p.num_query_heads / p.geom.num_kv_heads;
  const DecodePlan pl = make_decode_plan(p);
  if (!pl.tensor_cores) {
    b200::RowArgs a{};
    a.mode = b200::kRowBlockTable;
    a.q = p.query;
    a.q_srow = p.q_stride_row;
    a.q_shead = p.q_stride_head;
    a.query_rows = p.query_rows;
    a.kc = p.key_cache;
    a.vc = p.value_cache;
    a.layer = p.layer_idx;
    a.nb = p.geom.total_blocks;
    a.bs = p.geom.block_size;
    a.hkv = p.geom.num_kv_heads;
    a.head_dim = p.geom.head_dim;
    a.group = G;
    a.nchunks = (G + 7) / 8;
    a.bt = p.block_tables;
    a.bt_stride = p.block_table_stride;
    a.ctx_lens = p.context_lens;
    a.cu_q = nullptr;
    a.S = p.num_seqs;
    a.scale = p.scale;
    a.out = p.out;
    a.o_srow = p.o_stride_row;
    a.o_shead = p.o_stride_head;
    a.status = p.status_word;
    cudaError_t e = b200::launch_row(p.geom.dtype, a, p.num_seqs, st);
    if (e != cudaSuccess) return cuda_fail(e, "paged_decode(row)");
    return B200_OK;
  }
  if (workspace == nullptr || workspace_bytes < pl.total)
    return fail(B200_ERR_INVALID_ARGUMENT, "decode workspace too small");
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "decode workspace must be 256-byte aligned");
  char* ws = static_cast<char*>(workspace);
  auto* hdr = reinterpret_cast<b200::DecodeHeader*>(ws);
  auto* cu = reinterpret_cast<int32_t*>(ws + pl.off_cu);
  auto* work = reinterpret_cast<int2*>(ws + pl.off_work);
  auto* cnt = reinterpret_cast<int32_t*>(ws + pl.off_cnt);
  auto* lse = reinterpret_cast<float*>(ws + pl.off_lse);
  auto* po = reinterpret_cast<float*>(ws + pl.off_o);

  CUtensorMap km, vm;
  const int box_rows = p.geom.block_size >= 16 ? 16 : 8;
  rc = cache_tensor_map(p.key_cache, p.geom, box_rows, &km);
  if (rc != B200_OK) return rc;
  rc = cache_tensor_map(p.value_cache, p.geom, box_rows, &vm);
  if (rc != B200_OK) return rc;

  b200::PlanArgs pa{};
  pa.ctx_lens = p.context_lens;
  pa.query_rows = p.query_rows;
  pa.cu_q = cu_q;
  pa.S = p.num_seqs;
  pa.max_ctx = p.max_context_len;
  pa.split_tokens = pl.split_tokens;
  pa.items_per_split = pl.items_per_split;
  pa.hq = p.num_query_heads;
  pa.head_dim = p.geom.head_dim;
  pa.esize = esize_of(p.geom.dtype);
  pa.o_srow = p.o_stride_row;
  pa.o_shead = p.o_stride_head;
  pa.out = p.out;
  pa.status = p.status_word;
  pa.hdr = hdr;
  pa.cu_splits = cu;
  pa.work_sp = work;
  pa.counters = cnt;
  cudaError_t e = b200::launch_plan(pa, st);
  if (e != cudaSuccess) return cuda_fail(e, "decode plan");

  b200::DecodeArgs a{};
  a.q = p.query;
  a.q_srow = p.q_stride_row;
  a.q_shead = p.q_stride_head;
  a.query_rows = p.query_rows;
  a.cu_q = cu_q;
  a.layer = p.layer_idx;
  a.nb = p.geom.total_blocks;
  a.bs = p.geom.block_size;
  a.hkv = p.geom.num_kv_heads;
  a.hq = p.num_query_heads;
  a.group = G;
  a.nchunks = pl.nchunks;
  a.hpc = pl.hpc;
  a.bt = p.block_tables;
  a.bt_stride = p.block_table_stride;
  a.ctx_lens = p.context_lens;
  a.S = p.num_seqs;
  a.max_ctx = p.max_context_len;
  a.split_tokens = pl.split_tokens;
  a.scale_log2 = p.scale * b200::kLog2e;
  a.out = p.out;
  a.o_srow = p.o_stride_row;
  a.o_shead = p.o_stride_head;
  a.status = p.status_word;
  a.hdr = hdr;
  a.cu_splits = cu;
  a.work_sp = work;
  a.counters = cnt;
  a.part_lse = lse;
  a.part_o = po;
  const int64_t max_items = pl.max_splits * pl.items_per_split;
  e = b200::launch_decode_tc(p.geom.dtype, p.geom.head_dim, km, vm, a,
                             static_cast<int>(max_items < (1 << 30) ? max_items : (1 << 30)), st);
  if (e != cudaSuccess) return cuda_fail(e, "decode");
  return B200_OK;
}
}  // namespace

extern "C" {

int b200_paged_decode(const B200DecodeParams* pp, void* workspace, size_t workspace_bytes,
                      void* stream) {
  b200::NvtxRange nvtx_range("b200_paged_decode");
  if (pp == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null params");
  const B200DecodeParams& p = *pp;
  int rc = validate_geom(p.geom, p.layer_idx, p.num_query_heads);
  if (rc != B200_OK) return rc;
  if (p.num_seqs < 0) return fail(B200_ERR_INVALID_ARGUMENT, "num_seqs < 0");
  if (p.num_seqs == 0) return B200_OK;
  return run_decode(p, nullptr, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

// ---- prefill (ragged causal) ----------------------------------------------------------------

struct PrefillPlan {
  bool tensor_cores;
  bool split_decodes;  // one-token sequences go to the split-K decode kernel
  int tq;
  int64_t max_work;
  size_t decode_bytes, off_hdr, off_work, total;
};

// The decode leg of a mixed batch: every sequence, filtered on the device to those with one
// new token (their query row is cu_seqlens[s]).
static B200DecodeParams decode_leg(const B200PrefillParams& p) {
  B200DecodeParams d{};
  d.query = p.query;
  d.q_stride_row = p.q_stride_token;
  d.q_stride_head = p.q_stride_head;
  d.query_rows = nullptr;
  d.key_cache = p.key_cache;
  d.value_cache = p.value_cache;
  d.geom = p.geom;
  d.layer_idx = p.layer_idx;
  d.num_query_heads = p.num_query_heads;
  d.block_tables = p.block_tables;
  d.block_table_stride = p.block_table_stride;
  d.context_lens = p.context_lens;
  d.num_seqs = p.num_seqs;
  d.max_context_len = p.max_context_len;
  d.scale = p.scale;
  d.out = p.out;
  d.o_stride_row = p.o_stride_token;
  d.o_stride_head = p.o_stride_head;
  d.status_word = p.status_word;
  return d;
}

static PrefillPlan make_prefill_plan(const B200PrefillParams& p) {
  PrefillPlan pl{};
  const int G = p.num_query_heads / p.geom.num_kv_heads;
  const int es = esize_of(p.geom.dtype);
  pl.tensor_cores = (p.geom.dtype == B200_DTYPE_BF16 || p.geom.dtype == B200_DTYPE_F16) &&
                    (p.geom.head_dim == 64 || p.geom.head_dim == 128) &&
                    p.geom.block_size % 16 == 0 && G >= 1 && G <= 16 && 128 % G == 0 &&
                    reinterpret_cast<uintptr_t>(p.query) % 16 == 0 &&
                    (p.q_stride_token * es) % 16 == 0 && (p.q_stride_head * es) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(p.key_cache) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(p.value_cache) % 16 == 0 &&
                    static_cast<int64_t>(p.geom.num_layers) * p.geom.total_blocks *
                            p.geom.block_size < (int64_t(1) << 31);
  pl.tq = G > 0 ? 128 / G : 128;
  pl.max_work = static_cast<int64_t>(p.num_tokens) / (pl.tq > 0 ? pl.tq : 1) + p.num_seqs;
  const DecodePlan dpl = make_decode_plan(decode_leg(p));
  pl.split_decodes = pl.tensor_cores && dpl.tensor_cores;
  pl.decode_bytes = pl.split_decodes ? align256(dpl.total) : 0;
  pl.off_hdr = pl.decode_bytes;
  pl.off_work = pl.off_hdr + align256(sizeof(b200::PrefillHeader));
  pl.total = pl.tensor_cores ? pl.off_work + align256(pl.max_work * sizeof(int2)) : 0;
  return pl;
}

// Q (or any [token][head][dim] tensor of 2-byte elements) as a 4-D map: 64-element chunk,
// D/64 chunks, heads, tokens; box = one 128-byte row chunk x tq tokens, 128-byte swizzle.
static int query_tensor_map(const void* q, int64_t stride_tok, int64_t stride_head, int hq,
                            int ntok, int head_dim, int dtype, int tq, CUtensorMap* out) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[4] = {64, static_cast<cuuint64_t>(head_dim / 64),
                              static_cast<cuuint64_t>(hq), static_cast<cuuint64_t>(ntok)};
  const cuuint64_t strides[3] = {128, static_cast<cuuint64_t>(stride_head * 2),
                                 static_cast<cuuint64_t>(stride_tok * 2)};
  const cuuint32_t box[4] = {64, 1, 1, static_cast<cuuint32_t>(tq)};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = dtype == B200_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(out, dt, 4, const_cast<void*>(q), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200_ERR_CUDA, "cuTensorMapEncodeTiled (query) failed");
  return B200_OK;
}

size_t b200_paged_prefill_workspace_bytes(const B200PrefillParams* p) {
  if (p == nullptr || p->num_seqs <= 0 || p->geom.num_kv_heads <= 0 ||
      p->num_query_heads % p->geom.num_kv_heads != 0)
    return 0;
  return make_prefill_plan(*p).total;
}

int b200_paged_prefill(const B200PrefillParams* pp, void* workspace, size_t workspace_bytes,
                       void* stream) {
  b200::NvtxRange nvtx_range("b200_paged_prefill");
  if (pp == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null params");
  const B200PrefillParams& p = *pp;
  int rc = validate_geom(p.geom, p.layer_idx, p.num_query_heads);
  if (rc != B200_OK) return rc;
  if (p.num_seqs < 0 || p.num_tokens < 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "negative sizes");
  if (p.num_seqs == 0 || p.num_tokens == 0) return B200_OK;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int G = p.num_query_heads / p.geom.num_kv_heads;
  const PrefillPlan pl = make_prefill_plan(p);
  if (pl.tensor_cores && !g_force_cuda_core_prefill.load(std::memory_order_relaxed)) {
    if (workspace == nullptr || workspace_bytes < pl.total)
      return fail(B200_ERR_INVALID_ARGUMENT, "prefill workspace too small");
    if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
      return fail(B200_ERR_INVALID_ARGUMENT, "prefill workspace must be 256-byte aligned");
    char* ws = static_cast<char*>(workspace);
    if (pl.split_decodes) {
      rc = run_decode(decode_leg(p), p.cu_seqlens, ws, pl.decode_bytes, st);
      if (rc != B200_OK) return rc;
    }
    auto* hdr = reinterpret_cast<b200::PrefillHeader*>(ws + pl.off_hdr);
    auto* work = reinterpret_cast<int2*>(ws + pl.off_work);
    CUtensorMap qm, km, vm;
    rc = query_tensor_map(p.query, p.q_stride_token, p.q_stride_head, p.num_query_heads,
                          p.num_tokens, p.geom.head_dim, p.geom.dtype, pl.tq, &qm);
    if (rc != B200_OK) return rc;
    rc = cache_tensor_map(p.key_cache, p.geom, 16, &km);
    if (rc != B200_OK) return rc;
    rc = cache_tensor_map(p.value_cache, p.geom, 16, &vm);
    if (rc != B200_OK) return rc;
    // 0: one query tile per item (prefill.cu); 1: two tiles per item (prefill_q2.cu), which
    // takes query tiles in pairs (the work list, sized for single tiles, holds the pairs as
    // well); 2: two independent streams per CTA (prefill_ds.cu)
    const int kernel = g_prefill_kernel.load(std::memory_order_relaxed);
    const bool two_tiles = kernel == 1;
    b200::PrefillPlanArgs pa{};
    pa.cu_q = p.cu_seqlens;
    pa.ctx_lens = p.context_lens;
    pa.skip_single = pl.split_decodes ? 1 : 0;
    pa.S = p.num_seqs;
    pa.tq = two_tiles ? 2 * pl.tq : pl.tq;
    pa.hkv = p.geom.num_kv_heads;
    pa.max_work = static_cast<int32_t>(pl.max_work);
    pa.status = p.status_word;
    pa.hdr = hdr;
    pa.work = work;
    cudaError_t e = b200::launch_prefill_plan(pa, st);
    if (e != cudaSuccess) return cuda_fail(e, "prefill plan");
    b200::PrefillArgs a{};
    a.layer = p.layer_idx;
    a.nb = p.geom.total_blocks;
    a.bs = p.geom.block_size;
    a.hkv = p.geom.num_kv_heads;
    a.hq = p.num_query_heads;
    a.group = G;
    a.tq = pl.tq;
    a.bt = p.block_tables;
    a.bt_stride = p.block_table_stride;
    a.cu_q = p.cu_seqlens;
    a.ctx_lens = p.context_lens;
    a.S = p.num_seqs;
    a.scale_log2 = p.scale * b200::kLog2e;
    a.out = p.out;
    a.o_stok = p.o_stride_token;
    a.o_shead = p.o_stride_head;
    a.vec_out = (reinterpret_cast<uintptr_t>(p.out) % 16 == 0 && p.o_stride_token % 8 == 0 &&
                 p.o_stride_head % 8 == 0)
                    ? 1
                    : 0;
    a.status = p.status_word;
    a.hdr = hdr;
    a.work = work;
    const int64_t max_items = pl.max_work * p.geom.num_kv_heads;
    const int items = static_cast<int>(max_items < (1 << 30) ? max_items : (1 << 30));
    const int poly = g_prefill_poly_exp.load(std::memory_order_relaxed);
    if (kernel == 2)
      e = b200::launch_prefill_ds(p.geom.dtype, p.geom.head_dim, qm, km, vm, a, items, num_sms(),
                                  poly, st);
    else if (two_tiles)
      e = b200::launch_prefill_q2(p.geom.dtype, p.geom.head_dim, qm, km, vm, a, items, num_sms(),
                                  poly, st);
    else
      e = b200::launch_prefill_tc(p.geom.dtype, p.geom.head_dim, qm, km, vm, a, items, num_sms(),
                                  st);
    if (e != cudaSuccess) return cuda_fail(e, "prefill");
    return B200_OK;
  }
  b200::RowArgs a{};
  a.mode = b200::kRowBlockTable;
  a.q = p.query;
  a.q_srow = p.q_stride_token;
  a.q_shead = p.q_stride_head;
  a.kc = p.key_cache;
  a.vc = p.value_cache;
  a.layer = p.layer_idx;
  a.nb = p.geom.total_blocks;
  a.bs = p.geom.block_size;
  a.hkv = p.geom.num_kv_heads;
  a.head_dim = p.geom.head_dim;
  a.group = G;
  a.nchunks = (G + 7) / 8;
  a.bt = p.block_tables;
  a.bt_stride = p.block_table_stride;
  a.ctx_lens = p.context_lens;
  a.cu_q = p.cu_seqlens;
  a.S = p.num_seqs;
  a.scale = p.scale;
  a.out = p.out;
  a.o_srow = p.o_stride_token;
  a.o_shead = p.o_stride_head;
  a.status = p.status_word;
  cudaError_t e = b200::launch_row(p.geom.dtype, a, p.num_tokens, st);
  if (e != cudaSuccess) return cuda_fail(e, "paged_prefill(row)");
  return B200_OK;
}

void b200_set_prefill_poly_exp(int32_t mode) {
  g_prefill_poly_exp.store(mode < 0 || mode > 2 ? 1 : mode, std::memory_order_relaxed);
}

void b200_set_prefill_kernel(int32_t kernel) {
  g_prefill_kernel.store(kernel < 0 || kernel > 2 ? 1 : kernel, std::memory_order_relaxed);
}

void b200_set_prefill_cuda_cores(int32_t enable) {
  g_force_cuda_core_prefill.store(enable != 0, std::memory_order_relaxed);
}

// ---- reshape_and_cache ------------------------------------------------------------------------

int b200_reshape_and_cache(const void* key, int64_t k_stride_token, int64_t k_stride_head,
                           const void* value, int64_t v_stride_token, int64_t v_stride_head,
                           void* key_cache, void* value_cache, const B200CacheGeometry* geom,
                           int32_t layer_idx, const int64_t* slot_mapping, int32_t num_tokens,
                           int32_t* status_word, void* stream) {
  b200::NvtxRange nvtx_range("b200_reshape_and_cache");
  if (geom == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null geometry");
  const B200CacheGeometry& g = *geom;
  const int es = esize_of(g.dtype);
  if (es == 0) return fail(B200_ERR_UNSUPPORTED, "unsupported dtype");
  if (layer_idx < 0 || layer_idx >= g.num_layers)
    return fail(B200_ERR_INVALID_ARGUMENT, "layer_idx out of range");
  if (num_tokens < 0) return fail(B200_ERR_INVALID_ARGUMENT, "num_tokens < 0");
  if (num_tokens == 0) return B200_OK;
  b200::CacheWriteArgs a{};
  a.key = key;
  a.value = value;
  a.k_stok = k_stride_token * es;
  a.k_shead = k_stride_head * es;
  a.v_stok = v_stride_token * es;
  a.v_shead = v_stride_head * es;
  a.kc = key_cache;
  a.vc = value_cache;
  a.layer = layer_idx;
  a.nb = g.total_blocks;
  a.bs = g.block_size;
  a.hkv = g.num_kv_heads;
  a.head_bytes = static_cast<int64_t>(g.head_dim) * es;
  a.slots = slot_mapping;
  a.num_tokens = num_tokens;
  a.status = status_word;
  // widest vector that divides every address and stride
  uint64_t align = static_cast<uint64_t>(a.head_bytes) | static_cast<uint64_t>(a.k_stok) |
                   static_cast<uint64_t>(a.k_shead) | static_cast<uint64_t>(a.v_stok) |
                   static_cast<uint64_t>(a.v_shead) | reinterpret_cast<uintptr_t>(key) |
                   reinterpret_cast<uintptr_t>(value) | reinterpret_cast<uintptr_t>(key_cache) |
                   reinterpret_cast<uintptr_t>(value_cache);
  int vec = 16;
  while (vec > 2 && (align % vec) != 0) vec /= 2;
  if (align % vec != 0) return fail(B200_ERR_INVALID_ARGUMENT, "misaligned key/value rows");
  cudaError_t e = b200::launch_reshape_and_cache(a, vec, num_sms(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "reshape_and_cache");
  return B200_OK;
}

// ---- rotary + reshape_and_cache --------------------------------------------------------------

int b200_rope_reshape_and_cache(const void* qkv, int64_t qkv_stride_token, int32_t num_tokens,
                                int32_t num_query_heads, const int64_t* positions,
                                const float* inv_freq, void* q_out, int64_t q_out_stride_token,
                                void* key_cache, void* value_cache, const B200CacheGeometry* geom,
                                int32_t layer_idx, const int64_t* slot_mapping,
                                int32_t* status_word, void* stream) {
  b200::NvtxRange nvtx_range("b200_rope_reshape_and_cache");
  if (geom == nullptr) return fail(B200_ERR_INVALID_ARGUMENT, "null geometry");
  const B200CacheGeometry& g = *geom;
  if (esize_of(g.dtype) == 0) return fail(B200_ERR_UNSUPPORTED, "unsupported dtype");
  if (layer_idx < 0 || layer_idx >= g.num_layers)
    return fail(B200_ERR_INVALID_ARGUMENT, "layer_idx out of range");
  if (num_tokens < 0) return fail(B200_ERR_INVALID_ARGUMENT, "num_tokens < 0");
  if (g.head_dim % 2 != 0 || g.head_dim > 1024)
    return fail(B200_ERR_INVALID_ARGUMENT, "head_dim must be even and <= 1024");
  if (num_query_heads <= 0 || num_query_heads % g.num_kv_heads != 0)
    return fail(B200_ERR_INVALID_ARGUMENT, "num_query_heads must be a multiple of num_kv_heads");
  if (qkv_stride_token < static_cast<int64_t>(num_query_heads + 2 * g.num_kv_heads) * g.head_dim)
    return fail(B200_ERR_INVALID_ARGUMENT, "qkv_stride_token shorter than a q,k,v row");
  if (q_out_stride_token < static_cast<int64_t>(num_query_heads) * g.head_dim)
    return fail(B200_ERR_INVALID_ARGUMENT, "q_out_stride_token shorter than a q row");
  if (num_tokens == 0) return B200_OK;
  if (!qkv || !positions || !inv_freq || !q_out || !key_cache || !value_cache || !slot_mapping)
    return fail(B200_ERR_INVALID_ARGUMENT, "null pointer");
  b200::RopeCacheArgs a{};
  a.qkv = qkv;
  a.qkv_stok = qkv_stride_token;
  a.hq = num_query_heads;
  a.hkv = g.num_kv_heads;
  a.head_dim = g.head_dim;
  a.positions = positions;
  a.inv_freq = inv_freq;
  a.q_out = q_out;
  a.q_stok = q_out_stride_token;
  a.kc = key_cache;
  a.vc = value_cache;
  a.layer = layer_idx;
  a.nb = g.total_blocks;
  a.bs = g.block_size;
  a.slots = slot_mapping;
  a.num_tokens = num_tokens;
  a.status = status_word;
  cudaError_t e =
      b200::launch_rope_cache(a, g.dtype, num_sms(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope_reshape_and_cache");
  return B200_OK;
}

// ---- whole-block copy (swap out / swap in / copy before write) -------------------------------

namespace {
// The address the device uses for p: device and managed memory as is, page-locked host memory
// through its device mapping.  Pageable host memory (not reachable from the GPU) is rejected
// here, so no kernel is ever given it.
bool device_address(const void* p, const void** out) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  switch (at.type) {
    case cudaMemoryTypeDevice:
    case cudaMemoryTypeManaged:
      *out = p;
      return true;
    case cudaMemoryTypeHost:
      if (at.devicePointer == nullptr) return false;
      // p may point inside the registered range: keep its offset
      *out = static_cast<const char*>(at.devicePointer) +
             (static_cast<const char*>(p) - static_cast<const char*>(at.hostPointer));
      return true;
    default:
      return false;
  }
}
}  // namespace

int b200_copy_blocks(const void* src_key_cache, const void* src_value_cache,
                     const B200CacheGeometry* src_geom, void* dst_key_cache,
                     void* dst_value_cache, const B200CacheGeometry* dst_geom,
                     const int32_t* src_blocks, const int32_t* dst_blocks, int32_t num_blocks,
                     int32_t* status_word, void* stream) {
  b200::NvtxRange nvtx_range("b200_copy_blocks");
  if (src_geom == nullptr || dst_geom == nullptr)
    return fail(B200_ERR_INVALID_ARGUMENT, "null geometry");
  const B200CacheGeometry& s = *src_geom;
  const B200CacheGeometry& d = *dst_geom;
  if (s.num_layers != d.num_layers || s.block_size != d.block_size ||
      s.num_kv_heads != d.num_kv_heads || s.head_dim != d.head_dim || s.dtype != d.dtype)
    return fail(B200_ERR_INVALID_ARGUMENT,
                "source and destination caches differ in layers, block size, heads, head_dim or dtype");
  const int es = esize_of(s.dtype);
  if (es == 0) return fail(B200_ERR_UNSUPPORTED, "unsupported dtype");
  if (num_blocks < 0) return fail(B200_ERR_INVALID_ARGUMENT, "num_blocks < 0");
  if (num_blocks == 0) return B200_OK;
  if (!src_key_cache || !dst_key_cache || !src_blocks || !dst_blocks)
    return fail(B200_ERR_INVALID_ARGUMENT, "null pointer");
  const bool with_v = src_value_cache != nullptr;
  if (with_v != (dst_value_cache != nullptr))
    return fail(B200_ERR_INVALID_ARGUMENT, "value caches must be both given or both null");
  const void *sk, *dk, *sb, *db;
  const void *sv = nullptr, *dv = nullptr;
  if (!device_address(src_key_cache, &sk) || !device_address(dst_key_cache, &dk) ||
      (with_v && (!device_address(src_value_cache, &sv) || !device_address(dst_value_cache, &dv))) ||
      !device_address(src_blocks, &sb) || !device_address(dst_blocks, &db))
    return fail(B200_ERR_INVALID_ARGUMENT,
                "caches and block ids must be device memory or page-locked host memory");
  src_key_cache = sk;
  src_value_cache = sv;
  dst_key_cache = const_cast<void*>(dk);
  dst_value_cache = const_cast<void*>(dv);
  src_blocks = static_cast<const int32_t*>(sb);
  dst_blocks = static_cast<const int32_t*>(db);
  b200::BlockCopyArgs a{};
  a.src_k = src_key_cache;
  a.src_v = src_value_cache;
  a.dst_k = dst_key_cache;
  a.dst_v = dst_value_cache;
  a.layers = s.num_layers;
  a.kv_count = with_v ? 2 : 1;
  a.src_nb = s.total_blocks;
  a.dst_nb = d.total_blocks;
  a.block_bytes = static_cast<int64_t>(s.block_size) * s.num_kv_heads * s.head_dim * es;
  a.src_blocks = src_blocks;
  a.dst_blocks = dst_blocks;
  a.num_blocks = num_blocks;
  a.status = status_word;
  const uint64_t align = static_cast<uint64_t>(a.block_bytes) |
                         reinterpret_cast<uintptr_t>(src_key_cache) |
                         reinterpret_cast<uintptr_t>(src_value_cache) |
                         reinterpret_cast<uintptr_t>(dst_key_cache) |
                         reinterpret_cast<uintptr_t>(dst_value_cache);  // null is aligned
  int vec = 16;
  while (vec > 2 && (align % vec) != 0) vec /= 2;
  if (align % vec != 0) return fail(B200_ERR_INVALID_ARGUMENT, "misaligned cache pointers");
  cudaError_t e = b200::launch_copy_blocks(a, vec, num_sms(), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "copy_blocks");
  return B200_OK;
}

}  // extern "C"
