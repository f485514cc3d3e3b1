// runtime.cpp -- device-resident executor for .ennf models (load -> plan -> run).
//
// Mirrors the reference runtime's three stages (SPINN/run_time/spinn_runtime.c: spinn_load
// :21-124, spinn_plan :129-155, spinn_run :298-355) with every node on the GPU:
//
//  * load: parses the ENNF v2 image (header, dense WeightEntry table at header.reserved[0],
//    graph meta, node table, tensor meta; SPINN/ennf_def.h) into host tables.
//  * plan: assigns each activation a device layout (NHWC with the channel dimension padded
//    to a multiple of 4 for everything that feeds a convolution, row-major otherwise),
//    inserts the NCHW<->NHWC conversions at the graph edges, pre-transforms weights once
//    (K-major, tap-major, tf32-rounded; transposed Gemm operands; depthwise tap-major),
//    and packs every activation into ONE device arena with the reference planner's
//    best-fit/free-at-last-use algorithm (spinn_memory_planner.c:56-241) but 64-bit
//    offsets and 256-B alignment -- the reference clamps the arena to INT_MAX
//    (spinn_memory_planner.c:251) and stores 32-bit offsets (spinn_runtime.h:36-37).
//  * run: input H2D, the compiled step list (captured once into a CUDA graph), output D2H.
//
// Unlike the reference dispatcher (spinn_ops.c:224-226), an operator without a device
// implementation fails the plan instead of being skipped.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <functional>
#include <map>
#include <memory>
#include <vector>

#include "internal.h"

namespace spinn {

// ------------------------------------------------------------------ ENNF constants
enum : uint16_t {
  OP_ADD = 4, OP_DIV = 23, OP_MUL = 39, OP_SUB = 50, OP_CONV = 60, OP_AVGPOOL = 80, OP_GAP = 81, OP_MAXPOOL = 85,
  OP_BN = 100, OP_RELU = 130, OP_SIGMOID = 133, OP_GEMM = 160, OP_MATMUL = 161, OP_FLATTEN = 189,
  OP_IDENTITY = 193, OP_RESHAPE = 197, OP_SOFTMAX = 134, OP_CONCAT = 183, OP_RESIZE = 198, OP_SPLIT = 206,
  OP_TOPK = 210, OP_TRANSPOSE = 211
};
constexpr uint8_t kDtypeInt64 = 7;  // ENNF_TYPE_INT64 (SPINN/ennf_def.h)
constexpr uint32_t kMagic = 0x454E4E46;

#pragma pack(push, 1)
struct EnnfHeader {  // SPINN/ennf_def.h:70-95
  uint32_t magic;
  uint16_t vmaj, vmin;
  uint32_t num_nodes, num_tensors, num_weights, total_weight_bytes;
  uint16_t num_inputs, num_outputs, opset, flags;
  uint32_t graph_meta_offset, node_table_offset, tensor_meta_offset, weight_data_offset, string_table_offset;
  uint32_t reserved[3];
};
#pragma pack(pop)
static_assert(sizeof(EnnfHeader) == 64, "ENNF header is 64 bytes");

struct EnnfMeta {  // SPINN/ennf_def.h:130-139 as compiled (44 bytes)
  uint16_t tensor_id;
  uint8_t dtype, ndim;
  uint32_t dims[8];
  uint32_t elem_count;
  uint8_t is_weight, ref_count, pad[2];
};
static_assert(sizeof(EnnfMeta) == 44, "ENNF tensor meta is 44 bytes");

struct ConvParams {  // SPINN/ennf_op_params.h:23-31
  uint16_t kernel_shape[4], strides[4], pads[8], dilations[4], group;
  uint8_t auto_pad, fused_act;
};
static_assert(sizeof(ConvParams) == 44, "ENNF_ConvParams is 44 bytes");
struct PoolParams {  // ennf_op_params.h:45-56
  uint16_t kernel_shape[4], strides[4], pads[8], dilations[4];
  uint8_t auto_pad, ceil_mode, count_include_pad, storage_order;
  int32_t p;
};
static_assert(sizeof(PoolParams) == 48, "ENNF_PoolParams is 48 bytes");
struct GemmParams {  // ennf_op_params.h:134-140
  float alpha, beta;
  uint8_t transA, transB, reserved[2];
};
struct BnParams {
  float epsilon, momentum;
  uint8_t training_mode, reserved[3];
};

}  // namespace spinn

using namespace spinn;

struct TensorRec {
  uint16_t id = 0;
  uint8_t dtype = 0, ndim = 0;
  uint32_t dims[8] = {0};
  uint64_t elems = 0;
  bool is_weight = false;
  const float* host = nullptr;  // weights: into the file image
  uint64_t host_bytes = 0;
};

struct NodeRec {
  uint16_t op = 0;
  uint8_t flags = 0;
  std::vector<uint16_t> in, out;
  std::vector<uint8_t> params;
};

enum Layout { LAY_NONE = 0, LAY_ROW = 1, LAY_NHWC = 2 };

struct Buf {
  Layout lay = LAY_NONE;
  int n = 0, c = 0, h = 0, w = 0, cpad = 0;  // NHWC geometry
  uint64_t bytes = 0;
  int alias = -1;          // storage shared with this buffer index (resolved to a root)
  int external = 0;        // 1: lives outside the arena (graph input/output staging)
  int64_t offset = -1;
  float* ptr = nullptr;
  int first = -1, last = -1;  // step interval of use
};

struct StepRec {
  int kind = 0;
  int node = -1;
  uint16_t op = 0;
  double flops = 0;
  std::function<int(cudaStream_t)> run;
};

struct SpinnCudaModel {
  std::vector<uint8_t> image;
  EnnfHeader hdr{};
  std::vector<TensorRec> tensors;
  std::vector<NodeRec> nodes;
  std::vector<uint16_t> inputs, outputs;
  // plan
  bool planned = false;
  int device = -1;
  int flags = 0;
  cudaStream_t stream = nullptr;
  std::vector<Buf> bufs;           // [0, num_tensors) = ENNF tensors, then temporaries
  std::vector<int> in_buf, out_buf;  // NCHW staging buffer per graph input / output
  uint8_t* arena = nullptr;
  uint64_t arena_bytes = 0;
  float* wdev = nullptr;
  uint64_t wbytes = 0;
  int tc_layers = 0;               // tensor-core conv steps planned so far (tile walk direction)
  std::map<int, std::vector<int>> virt_cat;  // Concat outputs read in parts: tensor -> part buffers
  std::map<int, int> lazy_nchw;  // Reshape outputs gathered from NHWC: tensor -> viewed tensor
  std::map<int, int> b_trans;    // Transposes folded into a MatMul's B: tensor -> untransposed tensor
  float* splitk_ws = nullptr;      // split-K partial sums, shared by all steps (one stream)
  size_t splitk_bytes = 0;
  int* sk_flags = nullptr;         // stream-K handoff flags (kTcSkFlags ints), shared the same way
  bool sk_used = false;
  std::vector<float> whost;        // pre-transformed weights before upload
  std::vector<StepRec> steps;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t gexec = nullptr;
  cudaGraph_t pgraph = nullptr;      // same steps with an event between each (profiling)
  cudaGraphExec_t pgexec = nullptr;
  std::vector<cudaEvent_t> events;
  std::vector<float> step_ms;
  int kernels = 0;
  // pipelined submission (spinn_cuda_submit): input 0 alternates between its own staging
  // buffer (slot 0) and a second one (slot 1) read by a second captured graph, so the next
  // input's host copy (copy_stream) never touches the buffer the running graph reads
  cudaStream_t copy_stream = nullptr;
  void* alt_in = nullptr;                        // slot 1 input buffer
  cudaGraph_t graph_alt = nullptr;
  cudaGraphExec_t gexec_alt = nullptr;           // the step list reading alt_in
  cudaEvent_t in_ready[2] = {nullptr, nullptr};  // slot k filled (copy stream)
  cudaEvent_t in_free[2] = {nullptr, nullptr};   // the run reading slot k is done (model stream)
  uint64_t submitted = 0;
};

namespace spinn {
namespace {

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Records the split-K workspace a tcgen05 launch of this shape will want.
void note_ws(SpinnCudaModel* m, const TcGemmArgs& a) { m->splitk_bytes = std::max(m->splitk_bytes, tc_gemm_workspace_bytes(a)); }
int round4(int c) { return (c + 3) & ~3; }

// ------------------------------------------------------------------ load
int parse_image(SpinnCudaModel* m) {
  const auto& img = m->image;
  auto need = [&](uint64_t off, uint64_t len) { return off + len <= img.size(); };
  if (!need(0, sizeof(EnnfHeader))) {
    set_error("ennf: image shorter than the header");
    return SPINN_CUDA_EFORMAT;
  }
  std::memcpy(&m->hdr, img.data(), sizeof(EnnfHeader));
  const EnnfHeader& h = m->hdr;
  if (h.magic != kMagic) {
    set_error("ennf: bad magic 0x%08x", h.magic);
    return SPINN_CUDA_EFORMAT;
  }
  if (h.num_tensors == 0 || h.num_tensors > 65536 || h.num_nodes > 1000000) {
    set_error("ennf: implausible counts (%u tensors, %u nodes)", h.num_tensors, h.num_nodes);
    return SPINN_CUDA_EFORMAT;
  }
  // graph meta
  uint64_t p = h.graph_meta_offset;
  auto rd16 = [&](uint16_t* v) {
    if (!need(p, 2)) return false;
    std::memcpy(v, img.data() + p, 2);
    p += 2;
    return true;
  };
  uint16_t ni = 0, no = 0, v = 0;
  if (!rd16(&ni)) goto bad;
  for (int i = 0; i < ni; ++i) {
    if (!rd16(&v)) goto bad;
    m->inputs.push_back(v);
  }
  if (!rd16(&no)) goto bad;
  for (int i = 0; i < no; ++i) {
    if (!rd16(&v)) goto bad;
    m->outputs.push_back(v);
  }
  // tensor meta
  m->tensors.resize(h.num_tensors);
  for (uint32_t i = 0; i < h.num_tensors; ++i) {
    const uint64_t off = (uint64_t)h.tensor_meta_offset + (uint64_t)i * sizeof(EnnfMeta);
    if (!need(off, sizeof(EnnfMeta))) goto bad;
    EnnfMeta mt;
    std::memcpy(&mt, img.data() + off, sizeof(mt));
    if (mt.tensor_id >= h.num_tensors || mt.ndim > 8) goto bad;
    TensorRec& t = m->tensors[mt.tensor_id];
    t.id = mt.tensor_id;
    t.dtype = mt.dtype;
    t.ndim = mt.ndim;
    std::memcpy(t.dims, mt.dims, sizeof(t.dims));
    t.elems = 1;
    for (int d = 0; d < mt.ndim; ++d) t.elems *= mt.dims[d];
    t.is_weight = mt.is_weight != 0;
  }
  // weights (dense entry table, SPINN/run_time/spinn_runtime.c:363-407)
  for (uint32_t i = 0; i < h.num_tensors; ++i) {
    TensorRec& t = m->tensors[i];
    if (!t.is_weight) continue;
    const uint64_t eoff = (uint64_t)h.reserved[0] + (uint64_t)i * 16;
    if (!need(eoff, 16)) goto bad;
    uint32_t doff = 0, dsize = 0;
    std::memcpy(&doff, img.data() + eoff + 4, 4);
    std::memcpy(&dsize, img.data() + eoff + 8, 4);
    if (dsize == 0) continue;
    const uint64_t woff = (uint64_t)h.weight_data_offset + doff;
    if (!need(woff, dsize) || (woff & 3)) goto bad;
    t.host = reinterpret_cast<const float*>(img.data() + woff);
    t.host_bytes = dsize;
  }
  // nodes
  p = h.node_table_offset;
  for (uint32_t i = 0; i < h.num_nodes; ++i) {
    if (!need(p, 8)) goto bad;
    NodeRec n;
    const uint8_t* b = img.data() + p;
    std::memcpy(&n.op, b, 2);
    const uint8_t nin = b[2], nout = b[3];
    uint16_t psz;
    std::memcpy(&psz, b + 4, 2);
    n.flags = b[6];
    p += 8;
    for (int k = 0; k < nin; ++k) {
      if (!rd16(&v) || v >= h.num_tensors) goto bad;
      n.in.push_back(v);
    }
    for (int k = 0; k < nout; ++k) {
      if (!rd16(&v) || v >= h.num_tensors) goto bad;
      n.out.push_back(v);
    }
    if (!need(p, psz)) goto bad;
    n.params.assign(img.data() + p, img.data() + p + psz);
    p += psz;
    m->nodes.push_back(std::move(n));
  }
  for (auto id : m->inputs)
    if (id >= h.num_tensors) goto bad;
  for (auto id : m->outputs)
    if (id >= h.num_tensors) goto bad;
  return 0;
bad:
  set_error("ennf: truncated or inconsistent image");
  return SPINN_CUDA_EFORMAT;
}

// ------------------------------------------------------------------ plan helpers
struct Planner {
  SpinnCudaModel* m;
  int round_out;
  explicit Planner(SpinnCudaModel* mm) : m(mm), round_out(!(mm->flags & SPINN_CUDA_PLAN_NO_ROUND)) {}

  int new_buf(const Buf& b) {
    m->bufs.push_back(b);
    return (int)m->bufs.size() - 1;
  }
  int root(int b) const {
    while (m->bufs[b].alias >= 0) b = m->bufs[b].alias;
    return b;
  }
  void touch(int b, int step) {
    b = root(b);
    Buf& x = m->bufs[b];
    if (x.first < 0 || step < x.first) x.first = step;
    if (step > x.last) x.last = step;
  }
  const TensorRec& T(int id) const { return m->tensors[id]; }

  // weight staging: returns element offset into whost (256-B aligned)
  uint64_t wreserve(uint64_t elems) {
    uint64_t off = align_up(m->whost.size(), 64);
    m->whost.resize(off + elems, 0.0f);
    return off;
  }
};

// NHWC geometry of a 4-D tensor id.
void set_nhwc(Buf& b, const TensorRec& t) {
  b.lay = LAY_NHWC;
  b.n = t.dims[0];
  b.c = t.dims[1];
  b.h = t.dims[2];
  b.w = t.dims[3];
  b.cpad = round4(b.c);
  b.bytes = (uint64_t)b.n * b.h * b.w * b.cpad * 4;
}
// Bytes per element on the device: int64 tensors (TopK indices) keep 8, everything else is fp32.
uint64_t elem_bytes(const TensorRec& t) { return t.dtype == kDtypeInt64 ? 8 : 4; }

void set_row(Buf& b, const TensorRec& t) {
  b.lay = LAY_ROW;
  b.bytes = t.elems * elem_bytes(t);
}

// Best-fit allocation over the step intervals (reference algorithm, 64-bit).
int plan_arena(SpinnCudaModel* m, int nsteps, uint64_t budget) {
  struct Blk {
    uint64_t off, size;
  };
  std::vector<Blk> freel{{0, budget ? budget : ~0ull >> 1}};
  uint64_t peak = 0;
  std::vector<std::vector<int>> born(nsteps + 1), dies(nsteps + 1);
  // SPINN_CUDA_PLAN_KEEP: no buffer is released, so every intermediate keeps its value from
  // the last run (spinn_cuda_copy_tensor); the kernels and their tile plans do not change
  const bool keep = (m->flags & SPINN_CUDA_PLAN_KEEP) != 0;
  for (int i = 0; i < (int)m->bufs.size(); ++i) {
    Buf& b = m->bufs[i];
    if (b.alias >= 0 || b.external || b.bytes == 0 || b.first < 0) continue;
    born[b.first].push_back(i);
    dies[keep ? nsteps : b.last].push_back(i);
  }
  auto alloc = [&](uint64_t size, uint64_t* off) {
    size = align_up(size, 256);
    int best = -1;
    for (int k = 0; k < (int)freel.size(); ++k)
      if (freel[k].size >= size && (best < 0 || freel[k].size < freel[best].size)) best = k;
    if (best < 0) return false;
    *off = freel[best].off;
    if (freel[best].size == size)
      freel.erase(freel.begin() + best);
    else {
      freel[best].off += size;
      freel[best].size -= size;
    }
    return true;
  };
  auto release = [&](uint64_t off, uint64_t size) {
    size = align_up(size, 256);
    auto it = std::lower_bound(freel.begin(), freel.end(), off, [](const Blk& b, uint64_t o) { return b.off < o; });
    it = freel.insert(it, Blk{off, size});
    size_t k = it - freel.begin();
    if (k + 1 < freel.size() && freel[k].off + freel[k].size == freel[k + 1].off) {
      freel[k].size += freel[k + 1].size;
      freel.erase(freel.begin() + k + 1);
    }
    if (k > 0 && freel[k - 1].off + freel[k - 1].size == freel[k].off) {
      freel[k - 1].size += freel[k].size;
      freel.erase(freel.begin() + k);
    }
  };
  for (int s = 0; s <= nsteps; ++s) {
    for (int i : born[s]) {
      uint64_t off;
      if (!alloc(m->bufs[i].bytes, &off)) {
        set_error("plan: arena budget %llu bytes exceeded", (unsigned long long)budget);
        return SPINN_CUDA_ENOMEM;
      }
      m->bufs[i].offset = (int64_t)off;
      peak = std::max(peak, off + align_up(m->bufs[i].bytes, 256));
    }
    for (int i : dies[s]) release(m->bufs[i].offset, m->bufs[i].bytes);
  }
  m->arena_bytes = peak;
  return 0;
}

double conv_flops(const TensorRec& w, const TensorRec& y) {
  // 2 * N*OC*OH*OW * (C/g)*KH*KW
  return 2.0 * (double)y.elems * w.dims[1] * w.dims[2] * w.dims[3];
}

}  // namespace

// Whether node `ci` is a convolution that reads tensor `whole` (a channel Concat of `parts`) as
// its input through the tcgen05 path and can fetch it part by part: group 1, not Winograd, not
// the bottleneck-tail pattern's expand, every part a whole number of the tensor-core channel
// blocks (32 channels in tiled mode, the im2col block of the concatenated channels otherwise).
static bool concat_feeds_tc_conv(SpinnCudaModel* m, int ci, int whole, const std::vector<uint16_t>& parts) {
  const NodeRec& nd = m->nodes[ci];
  if (nd.op != OP_CONV || nd.in.size() < 2 || nd.in[0] != whole) return false;
  for (size_t i = 1; i < nd.in.size(); ++i)
    if (nd.in[i] == whole) return false;
  ConvParams cp{};
  if (nd.params.size() >= sizeof(ConvParams)) std::memcpy(&cp, nd.params.data(), sizeof(cp));
  const TensorRec& W = m->tensors[nd.in[1]];
  const TensorRec& X = m->tensors[whole];
  const TensorRec& Y = m->tensors[nd.out[0]];
  if (W.ndim != 4 || !W.host || X.ndim != 4 || Y.ndim != 4) return false;
  const int G = cp.group > 0 ? cp.group : 1;
  const int KH = cp.kernel_shape[0] ? cp.kernel_shape[0] : (int)W.dims[2];
  const int KW = cp.kernel_shape[1] ? cp.kernel_shape[1] : (int)W.dims[3];
  const int SH = cp.strides[0] ? cp.strides[0] : 1, SW = cp.strides[1] ? cp.strides[1] : 1;
  const int DH = cp.dilations[0] ? cp.dilations[0] : 1, DW = cp.dilations[1] ? cp.dilations[1] : 1;
  if (G != 1 || cp.auto_pad != 0) return false;
  if ((m->flags & SPINN_CUDA_PLAN_WINOGRAD) && KH == 3 && KW == 3 && SH == 1 && SW == 1 && DH == 1 && DW == 1)
    return false;
  const int act = cp.fused_act;
  if ((act == 4 || act == 5) && KH == 1 && KW == 1) return false;  // may become a bottleneck-tail expand
  const int C = (int)X.dims[1];
  if (C % 4) return false;
  // a pointwise convolution reads A in 32-column tiled boxes when every part is a multiple of
  // 32 channels (conv_reads_parts_tiled), otherwise through the im2col path with the channel
  // block of the concatenated channels
  int cb = 32;
  for (int c : {32, 16, 8, 4})
    if (C % c == 0) {
      cb = c;
      break;
    }
  for (auto id : parts) {
    const TensorRec& t = m->tensors[id];
    if (t.ndim != 4 || (int)t.dims[1] % cb) return false;
  }
  return true;
}

// Whether a pointwise convolution reading a Concat in parts can use tiled A boxes (32 columns).
static bool conv_reads_parts_tiled(const SpinnCudaModel* m, const std::vector<int>& part_bufs) {
  for (int b : part_bufs)
    if (m->bufs[b].cpad % 32) return false;
  return true;
}

// Whether node `ri` is a Reshape [N,C,H,W] -> [N,C,H*W] whose only reader is a Concat along
// the last axis of 3-D tensors with at most four inputs.  Such a Reshape of an NHWC tensor is
// left as a view: the Concat reads the NHWC data transposed (launch_gather_rows), so the NCHW
// copy that the Reshape would otherwise need is never made.
static bool reshape_feeds_gather(const SpinnCudaModel* m, int ri, const std::vector<int>& readers,
                                 const std::vector<int>& reader_node) {
  const NodeRec& nd = m->nodes[ri];
  if (nd.op != OP_RESHAPE || nd.in.empty() || nd.out.size() != 1) return false;
  const TensorRec& X = m->tensors[nd.in[0]];
  const int yid = nd.out[0];
  const TensorRec& Y = m->tensors[yid];
  if (X.ndim != 4 || Y.ndim != 3 || Y.dims[0] != X.dims[0] || Y.dims[1] != X.dims[1] ||
      (uint64_t)Y.dims[2] != (uint64_t)X.dims[2] * X.dims[3] || X.dtype == kDtypeInt64)
    return false;
  if (readers[yid] != 1 || reader_node[yid] <= ri) return false;
  const NodeRec& cat = m->nodes[reader_node[yid]];
  if (cat.op != OP_CONCAT || cat.in.size() > 4 || cat.out.size() != 1) return false;
  int axis = 1;
  if (cat.params.size() >= 4) std::memcpy(&axis, cat.params.data(), 4);
  if (axis != 2 && axis != -1) return false;
  if (m->tensors[cat.out[0]].ndim != 3) return false;
  int uses = 0;
  for (auto id : cat.in) uses += id == yid;
  return uses == 1;
}

// ------------------------------------------------------------------ plan
static int compile_model(SpinnCudaModel* m, uint64_t budget) {
  Planner P(m);
  const int nt = (int)m->tensors.size();
  m->bufs.assign(nt, Buf());
  std::vector<int> produced(nt, 0);
  int step = 0;
  // pass-1 records: lambdas that build the closure once pointers are known
  std::vector<std::function<int(StepRec&)>> builders;
  // readers of each tensor (graph outputs count as one more); a channel Concat whose only
  // reader is a tensor-core convolution is not materialised: the convolution reads its parts
  std::vector<int> readers(nt, 0);
  std::vector<int> reader_node(nt, -1);
  for (int ni = 0; ni < (int)m->nodes.size(); ++ni)
    for (auto id : m->nodes[ni].in) {
      ++readers[id];
      reader_node[id] = ni;
    }
  for (auto id : m->outputs) ++readers[id];
  std::map<int, std::vector<int>> virt_cat;  // concat tensor -> NHWC buffers of its parts
  std::map<int, int> lazy_nchw;  // Reshape output -> the NHWC tensor it views (read by a gathering Concat)
  std::map<int, int> b_trans;    // Transpose output read only as a MatMul's B -> the untransposed tensor

  auto add_step = [&](int node, uint16_t op, int kind, double flops, std::function<int(StepRec&)> b) {
    StepRec s;
    s.node = node;
    s.op = op;
    s.kind = kind;
    s.flops = flops;
    m->steps.push_back(std::move(s));
    builders.push_back(std::move(b));
    return step++;
  };

  // graph inputs: NCHW staging buffers outside the arena; the tensor aliases its staging and
  // consumers convert on demand (ensure_nhwc, or the space-to-depth stem below)
  for (size_t i = 0; i < m->inputs.size(); ++i) {
    const int id = m->inputs[i];
    const TensorRec& t = m->tensors[id];
    Buf st;
    st.lay = LAY_ROW;
    st.bytes = t.elems * elem_bytes(t);
    st.external = 1;
    const int sb = P.new_buf(st);
    m->in_buf.push_back(sb);
    m->bufs[id] = m->bufs[sb];
    m->bufs[id].external = 0;
    m->bufs[id].alias = sb;
    produced[id] = 1;
  }

  std::map<int, int> nhwc_of;  // row-major 4-D tensor id -> its NHWC copy
  auto ensure_nhwc = [&](int id, int node) -> int {
    // returns a buffer index holding tensor `id` in NHWC layout
    Buf& b = m->bufs[id];
    if (b.lay == LAY_NHWC) return id;
    const TensorRec& t = m->tensors[id];
    if (t.ndim != 4) return -1;
    auto it = nhwc_of.find(id);
    if (it != nhwc_of.end()) return it->second;
    Buf nb;
    set_nhwc(nb, t);
    const int tb = P.new_buf(nb);
    const int rnd = P.round_out;
    const int s = add_step(node, 0, 7, 0, [m, id, tb, rnd](StepRec& r) {
      const Buf& x = m->bufs[id];
      const Buf& y = m->bufs[tb];
      r.run = [&x, &y, rnd](cudaStream_t st) {
        return launch_nchw_to_nhwc(x.ptr, y.ptr, y.n, y.c, y.h, y.w, y.cpad, st, rnd);
      };
      return 0;
    });
    P.touch(id, s);
    P.touch(tb, s);
    nhwc_of[id] = tb;
    return tb;
  };
  auto ensure_row = [&](int id, int node) -> int {
    Buf& b = m->bufs[id];
    if (b.lay == LAY_ROW) return id;
    const TensorRec& t = m->tensors[id];
    Buf nb;
    set_row(nb, t);
    const int tb = P.new_buf(nb);
    const int s = add_step(node, 0, 7, 0, [m, id, tb](StepRec& r) {
      const Buf& x = m->bufs[id];
      const Buf& y = m->bufs[tb];
      r.run = [&x, &y](cudaStream_t st) { return launch_nhwc_to_nchw(x.ptr, y.ptr, x.n, x.c, x.h, x.w, x.cpad, st); };
      return 0;
    });
    P.touch(id, s);
    P.touch(tb, s);
    return tb;
  };

  for (int ni = 0; ni < (int)m->nodes.size(); ++ni) {
    const NodeRec& nd = m->nodes[ni];
    for (auto id : nd.in) {
      const TensorRec& t = m->tensors[id];
      if (!t.is_weight && !produced[id] && t.elems > 0) {
        set_error("plan: node %d (op %d) reads tensor %d before it is produced", ni, nd.op, id);
        return SPINN_CUDA_EFORMAT;
      }
    }
    switch (nd.op) {
      case OP_CONV: {
        if (nd.in.size() < 2 || nd.out.empty()) {
          set_error("plan: Conv node %d has too few inputs", ni);
          return SPINN_CUDA_EFORMAT;
        }
        ConvParams cp{};
        if (nd.params.size() >= sizeof(ConvParams)) std::memcpy(&cp, nd.params.data(), sizeof(cp));
        const int act = cp.fused_act;
        const bool has_res = act == 4 || act == 5;
        const int n_real = has_res ? (int)nd.in.size() - 1 : (int)nd.in.size();
        const TensorRec& X = m->tensors[nd.in[0]];
        const TensorRec& W = m->tensors[nd.in[1]];
        const TensorRec& Y = m->tensors[nd.out[0]];
        if (X.ndim != 4 || W.ndim != 4 || Y.ndim != 4 || !W.host) {
          set_error("plan: Conv node %d needs 4-D X/W/Y and constant weights", ni);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        const int N = X.dims[0], C = X.dims[1], H = X.dims[2], Wd = X.dims[3];
        const int OC = W.dims[0], KC = W.dims[1];
        int KH = W.dims[2], KW = W.dims[3], SH = 1, SW = 1, PH = 0, PW = 0, DH = 1, DW = 1, G = 1;
        if (nd.params.size() >= sizeof(ConvParams)) {
          if (cp.group > 0) G = cp.group;
          if (cp.kernel_shape[0]) KH = cp.kernel_shape[0];
          if (cp.kernel_shape[1]) KW = cp.kernel_shape[1];
          if (cp.strides[0]) SH = cp.strides[0];
          if (cp.strides[1]) SW = cp.strides[1];
          if (cp.dilations[0]) DH = cp.dilations[0];
          if (cp.dilations[1]) DW = cp.dilations[1];
          PH = cp.pads[0];
          PW = cp.pads[1];
          if (cp.auto_pad == 1 || cp.auto_pad == 2) {  // SAME (conv2d.c:134-141)
            int ph = ((int)Y.dims[2] - 1) * SH + KH - H;
            if (ph < 0) ph = 0;
            int pw = ((int)Y.dims[3] - 1) * SW + KW - Wd;
            if (pw < 0) pw = 0;
            PH = cp.auto_pad == 1 ? ph / 2 : (ph + 1) / 2;
            PW = cp.auto_pad == 1 ? pw / 2 : (pw + 1) / 2;
          }
        }
        const int OH = Y.dims[2], OW = Y.dims[3];
        if ((int)Y.dims[1] != OC || (int)Y.dims[0] != N || C != KC * G || OC % G) {
          set_error("plan: Conv node %d shape mismatch", ni);
          return SPINN_CUDA_EFORMAT;
        }
        // Space-to-depth stem: a stride-2 convolution over a graph input with <= 4 channels is
        // run as a stride-1, pad-0 convolution over
        //   X'[n][i][j][(dy*2+dx)*4 + c] = x[n][c][2i+dy-PH][2j+dx-PW]     (16 channels)
        // with ceil(KH/2) x ceil(KW/2) taps and W'[o][ky][kx][dy][dx][c] = W[o][c][2ky+dy][2kx+dx].
        // Same sums; the tensor-core tile then takes 16 channels per tap instead of 4.
        bool is_input = false;
        for (auto id : m->inputs) is_input |= (id == nd.in[0]);
        const bool s2d = G == 1 && SH == 2 && SW == 2 && DH == 1 && DW == 1 && C <= 4 && KH >= 2 && KW >= 2 &&
                         is_input && m->bufs[nd.in[0]].lay == LAY_ROW;
        int xb;
        int Hc = H, Wc = Wd, Cc = round4(C), KHc = KH, KWc = KW, SHc = SH, SWc = SW, PHc = PH, PWc = PW, DHc = DH,
            DWc = DW;
        if (s2d) {
          KHc = (KH + 1) / 2;
          KWc = (KW + 1) / 2;
          Hc = OH + KHc - 1;
          Wc = OW + KWc - 1;
          Cc = 16;
          SHc = SWc = 1;
          PHc = PWc = 0;
          Buf sb;
          sb.lay = LAY_NHWC;
          sb.n = N;
          sb.c = Cc;
          sb.cpad = Cc;
          sb.h = Hc;
          sb.w = Wc;
          sb.bytes = (uint64_t)N * Hc * Wc * Cc * 4;
          xb = P.new_buf(sb);
          const int src = nd.in[0];
          const int rnd_in = P.round_out;
          const int s = add_step(ni, 0, 7, 0, [=](StepRec& r) {
            const Buf* x = &m->bufs[src];
            const Buf* y = &m->bufs[xb];
            r.run = [=](cudaStream_t st) {
              return launch_space_to_depth2(x->ptr, y->ptr, N, C, H, Wd, Hc, Wc, PH, PW, st, rnd_in);
            };
            return 0;
          });
          P.touch(src, s);
          P.touch(xb, s);
        } else {
          xb = ensure_nhwc(nd.in[0], ni);
        }
        int rb = -1;
        if (has_res) {
          rb = ensure_nhwc(nd.in.back(), ni);
          if (rb < 0) {
            set_error("plan: Conv node %d residual is not 4-D", ni);
            return SPINN_CUDA_EUNSUPPORTED;
          }
        }
        const int yb = nd.out[0];
        set_nhwc(m->bufs[yb], Y);
        const int cpad = round4(C), ocpad = round4(OC);
        const TensorRec* B = (n_real > 2 && m->tensors[nd.in[2]].host) ? &m->tensors[nd.in[2]] : nullptr;
        const double fl = conv_flops(W, Y);
        const int rnd = P.round_out;
        const bool wino = (m->flags & SPINN_CUDA_PLAN_WINOGRAD) && G == 1 && !s2d && KH == 3 && KW == 3 && SH == 1 &&
                          SW == 1 && DH == 1 && DW == 1;
        // Bottleneck tail: this 1x1 expand with a fused residual, followed by a 1x1 reduce of
        // its output (the next block's first convolution), runs as one kernel that keeps y's
        // chunks in shared memory for the reduce (tail.cu) -- when there are rows enough for
        // eight waves of 128-row tiles (with fewer, the separate launches spread their more
        // numerous, narrower tiles better: ResNet-101 at batch 32, 5.3 waves, was 0.6% slower
        // fused, at 64 and 256 0.9% and 1.4% faster) and the expand's input is at most 128
        // channels wide.  Measured at batch 256: the 64 -> 256 -> 64 ends of the 56x56 stage
        // take 397-422 us fused against 457-498 us as two launches; 128 -> 512 -> 128 at 28x28
        // ties per launch (252 vs 250 us) and saves 0.07 ms over the step; 256 -> 1024 -> 256 at
        // 14x14 loses: 180 vs 149 us per pair of layers, 191 us on CTA pairs (half the weight
        // bytes per SM), and 64-column chunks through two y buffers made the step 15% slower;
        // its 128-row tiles stream ~3.5 MB each through shared memory, eight chunks in a row.
        const NodeRec* nb = ni + 1 < (int)m->nodes.size() ? &m->nodes[ni + 1] : nullptr;
        int oc2 = 0, act2 = 0;
        const TensorRec* W2 = nullptr;
        const TensorRec* B2 = nullptr;
        bool tail = false;
        if (!(m->flags & SPINN_CUDA_PLAN_NO_FUSE) && !virt_cat.count(nd.in[0]) && !wino && !s2d && G == 1 &&
            KH == 1 && KW == 1 && SH == 1 &&
            SW == 1 && PH == 0 && PW == 0 && OH == H && OW == Wd && has_res && n_real == 3 && C % 32 == 0 &&
            C <= 128 && OC % 128 == 0 && nb && nb->op == OP_CONV && nb->in.size() == 3 && nb->out.size() == 1 &&
            nb->in[0] == nd.out[0] && (long)N * H * Wd >= 8L * 128 * sm_count(m->device)) {
          ConvParams c2{};
          if (nb->params.size() >= sizeof(ConvParams)) std::memcpy(&c2, nb->params.data(), sizeof(c2));
          W2 = &m->tensors[nb->in[1]];
          B2 = &m->tensors[nb->in[2]];
          const TensorRec& Y2 = m->tensors[nb->out[0]];
          act2 = c2.fused_act;
          const int g2 = c2.group > 0 ? c2.group : 1;
          oc2 = W2->ndim == 4 ? (int)W2->dims[0] : 0;
          tail = (act2 == 0 || act2 == 1) && g2 == 1 && W2->ndim == 4 && W2->host && B2->host && W2->dims[1] == (uint32_t)OC &&
                 W2->dims[2] == 1 && W2->dims[3] == 1 && (c2.kernel_shape[0] <= 1) && (c2.kernel_shape[1] <= 1) &&
                 (c2.strides[0] <= 1) && (c2.strides[1] <= 1) && c2.pads[0] == 0 && c2.pads[1] == 0 &&
                 c2.pads[2] == 0 && c2.pads[3] == 0 && c2.auto_pad == 0 && oc2 % 32 == 0 && oc2 >= 32 &&
                 oc2 <= 256 && Y2.ndim == 4 && Y2.dims[1] == (uint32_t)oc2 && Y2.dims[2] == (uint32_t)OH &&
                 Y2.dims[3] == (uint32_t)OW;
        }
        if (tail) {
          const TensorRec* B = (n_real > 2 && m->tensors[nd.in[2]].host) ? &m->tensors[nd.in[2]] : nullptr;
          const int xb = ensure_nhwc(nd.in[0], ni);
          const int rb = ensure_nhwc(nd.in.back(), ni);
          if (xb < 0 || rb < 0) {
            set_error("plan: Conv node %d inputs are not 4-D", ni);
            return SPINN_CUDA_EUNSUPPORTED;
          }
          const int yb = nd.out[0], tb = nb->out[0];
          set_nhwc(m->bufs[yb], Y);
          set_nhwc(m->bufs[tb], m->tensors[tb]);
          // weights K-major, tf32-rounded: W3 [OC][C], W1 [oc2][OC]
          const uint64_t w3 = P.wreserve((uint64_t)OC * C), w1 = P.wreserve((uint64_t)oc2 * OC);
          for (uint64_t i = 0; i < (uint64_t)OC * C; ++i) m->whost[w3 + i] = host_round_tf32(W.host[i]);
          for (uint64_t i = 0; i < (uint64_t)oc2 * OC; ++i) m->whost[w1 + i] = host_round_tf32(W2->host[i]);
          const uint64_t b3 = P.wreserve(OC), b1 = P.wreserve(oc2);
          for (int o = 0; o < OC; ++o) m->whost[b3 + o] = B ? B->host[o] : 0.0f;
          for (int o = 0; o < oc2; ++o) m->whost[b1 + o] = B2->host[o];
          const double fl = conv_flops(W, Y) + conv_flops(*W2, m->tensors[tb]);
          const int rnd = P.round_out, M = N * H * Wd, n1 = OC, k1 = C, n2 = oc2, ae = act, ar = act2;
          const int s = add_step(ni, OP_CONV, 9, fl, [=](StepRec& r) {
            const Buf* xbp = &m->bufs[xb];
            const Buf* rbp = &m->bufs[rb];
            const Buf* ybp = &m->bufs[yb];
            const Buf* tbp = &m->bufs[tb];
            m->tc_layers |= 1;  // the next layer walks its tiles from the end, where this one stopped
            r.run = [=](cudaStream_t st) {
              TailArgs a;
              a.t2 = xbp->ptr;
              a.x = rbp->ptr;
              a.w3 = m->wdev + w3;
              a.w1 = m->wdev + w1;
              a.b3 = m->wdev + b3;
              a.b1 = m->wdev + b1;
              a.y = ybp->ptr;
              a.t = tbp->ptr;
              a.M = M;
              a.k1 = k1;
              a.n1 = n1;
              a.n2 = n2;
              a.kpad3 = k1;
              a.kpad1 = n1;
              a.act_e = ae;
              a.act_r = ar;
              a.round_out = rnd;
              return tail_fused_launch(a, st);
            };
            return 0;
          });
          P.touch(xb, s);
          P.touch(rb, s);
          P.touch(yb, s);
          P.touch(tb, s);
          produced[yb] = 1;
          produced[tb] = 1;
          ++ni;  // the reduce node is part of this step
          break;
        }
        if (wino) {
          // Winograd F(4x4,3x3): transforms in HBM, 36 tcgen05 GEMMs (winograd.cu)
          const int kpad = tc_num_kb(3 * cpad) * 32;
          const uint64_t woff = P.wreserve((uint64_t)36 * ocpad * kpad);
          winograd_f43_weights(W.host, OC, C, cpad, ocpad, kpad, &m->whost[woff]);
          uint64_t boff = ~0ull;
          if (B) {
            boff = P.wreserve(ocpad);
            for (int o = 0; o < OC; ++o) m->whost[boff + o] = B->host[o];
          }
          const long tiles = winograd_tiles(N, OH, OW);
          Buf vb, mb;
          vb.lay = mb.lay = LAY_ROW;
          vb.bytes = (uint64_t)36 * tiles * 3 * cpad * 4;
          mb.bytes = (uint64_t)36 * tiles * ocpad * 4;
          const int vbi = P.new_buf(vb), mbi = P.new_buf(mb);
          const int s = add_step(ni, OP_CONV, 8, fl, [=](StepRec& r) {
            const Buf* xbp = &m->bufs[xb];
            const Buf* ybp = &m->bufs[yb];
            const Buf* rbp = rb >= 0 ? &m->bufs[rb] : nullptr;
            const Buf* vp = &m->bufs[vbi];
            const Buf* mp = &m->bufs[mbi];
            r.run = [=](cudaStream_t st) {
              WinogradArgs a;
              a.x = xbp->ptr;
              a.n = N;
              a.h = H;
              a.w = Wd;
              a.cpad = cpad;
              a.oh = OH;
              a.ow = OW;
              a.ph = PH;
              a.pw = PW;
              a.u = m->wdev + woff;
              a.ocpad = ocpad;
              a.kpad = kpad;
              a.v = vp->ptr;
              a.m = mp->ptr;
              a.bias = boff != ~0ull ? m->wdev + boff : nullptr;
              a.res = rbp ? rbp->ptr : nullptr;
              a.y = ybp->ptr;
              a.act = act;
              a.round_out = rnd;
              return winograd_f43_run(a, st);
            };
            return 0;
          });
          P.touch(xb, s);
          P.touch(yb, s);
          P.touch(vbi, s);
          P.touch(mbi, s);
          if (rb >= 0) P.touch(rb, s);
        } else if (G == 1) {
          // tcgen05 implicit GEMM: weights [ocpad][kpad], k = (r*KWc + s)*Cc + c
          const int K = KHc * KWc * Cc;
          const int kpad = tc_num_kb(K) * 32;
          const uint64_t woff = P.wreserve((uint64_t)ocpad * kpad);
          for (int o = 0; o < OC; ++o)
            for (int c = 0; c < C; ++c)
              for (int r = 0; r < KH; ++r)
                for (int s = 0; s < KW; ++s) {
                  const float v = host_round_tf32(W.host[(((uint64_t)o * C + c) * KH + r) * KW + s]);
                  const uint64_t k = s2d ? (uint64_t)((r / 2) * KWc + s / 2) * Cc + ((r % 2) * 2 + s % 2) * 4 + c
                                         : (uint64_t)(r * KW + s) * cpad + c;
                  m->whost[woff + (uint64_t)o * kpad + k] = v;
                }
          uint64_t boff = ~0ull;
          if (B) {
            boff = P.wreserve(ocpad);
            for (int o = 0; o < OC; ++o) m->whost[boff + o] = B->host[o];
          }
          const std::vector<int> vparts = virt_cat.count(nd.in[0]) ? virt_cat[nd.in[0]] : std::vector<int>{};
          const int s = add_step(ni, OP_CONV, 1, fl, [=](StepRec& r) {
            TcGemmArgs a;
            a.a_mode = 0;
            a.n = N;
            a.h = Hc;
            a.w = Wc;
            a.cpad = Cc;
            a.kh = KHc;
            a.kw = KWc;
            a.sh = SHc;
            a.sw = SWc;
            a.ph = PHc;
            a.pw = PWc;
            a.dh = DHc;
            a.dw = DWc;
            a.oh = OH;
            a.ow = OW;
            a.M = N * OH * OW;
            a.K = KHc * KWc * Cc;
            a.kpad = kpad;
            a.N = ocpad;
            a.ldy = ocpad;
            a.ldr = ocpad;
            a.act = act;
            a.round_out = rnd;
            a.reverse = (m->tc_layers++) & 1;
            if (KHc == 1 && KWc == 1 && SHc == 1 && SWc == 1 && PHc == 0 && PWc == 0 && OH == Hc && OW == Wc &&
                (vparts.empty() || conv_reads_parts_tiled(m, vparts))) {
              // a pointwise conv over NHWC rows is a plain GEMM: tiled TMA boxes for A
              a.a_mode = 1;
              a.K = Cc;
              a.lda = Cc;
            }
            const Buf* xbp = &m->bufs[xb];
            const Buf* ybp = &m->bufs[yb];
            const Buf* rbp = rb >= 0 ? &m->bufs[rb] : nullptr;
            std::vector<const Buf*> xparts;  // a Concat read in parts
            if (vparts.size() > 1) {
              a.nparts = (int)vparts.size();
              int c0 = 0;
              for (int i = 0; i < a.nparts; ++i) {
                const Buf* pbuf = &m->bufs[vparts[i]];
                xparts.push_back(pbuf);
                a.xpart[i] = pbuf->ptr;
                a.part_c0[i] = c0;
                a.part_cpad[i] = pbuf->cpad;
                c0 += pbuf->cpad;
              }
            }
            // stream-K schedules for convolutions whose tiles leave the last wave short
            // (SPINN_NO_SK=1 turns them off, for comparisons)
            a.sk = getenv("SPINN_NO_SK") == nullptr;
            m->sk_used |= a.sk != 0;
            note_ws(m, a);
            r.run = [m, a, xbp, ybp, rbp, woff, boff, xparts](cudaStream_t st) mutable {
              a.ws = m->splitk_ws;
              a.ws_bytes = m->splitk_bytes;
              a.sk_flags = m->sk_flags;
              for (size_t i = 0; i < xparts.size(); ++i) a.xpart[i] = xparts[i]->ptr;
              a.x = xbp->ptr;
              a.y = ybp->ptr;
              a.res = rbp ? rbp->ptr : nullptr;
              a.wt = m->wdev + woff;
              a.bias = boff != ~0ull ? m->wdev + boff : nullptr;
              return tc_gemm_launch(a, st);
            };
            return 0;
          });
          P.touch(xb, s);
          for (int b : vparts) P.touch(b, s);
          P.touch(yb, s);
          if (rb >= 0) P.touch(rb, s);
        } else if (G == C && G == OC) {
          // depthwise: weights [KH*KW][ocpad]
          const uint64_t woff = P.wreserve((uint64_t)KH * KW * ocpad);
          for (int o = 0; o < OC; ++o)
            for (int t = 0; t < KH * KW; ++t) m->whost[woff + (uint64_t)t * ocpad + o] = W.host[(uint64_t)o * KH * KW + t];
          const uint64_t boff = P.wreserve(ocpad);
          if (B)
            for (int o = 0; o < OC; ++o) m->whost[boff + o] = B->host[o];
          const int s = add_step(ni, OP_CONV, 3, fl, [=](StepRec& r) {
            const Buf* xbp = &m->bufs[xb];
            const Buf* ybp = &m->bufs[yb];
            const Buf* rbp = rb >= 0 ? &m->bufs[rb] : nullptr;
            r.run = [=](cudaStream_t st) {
              return launch_depthwise_nhwc(xbp->ptr, m->wdev + woff, m->wdev + boff, rbp ? rbp->ptr : nullptr, ybp->ptr,
                                           N, H, Wd, ocpad, OH, OW, KH, KW, SH, SW, PH, PW, DH, DW, act, rnd, st);
            };
            return 0;
          });
          P.touch(xb, s);
          P.touch(yb, s);
          if (rb >= 0) P.touch(rb, s);
        } else {
          const int cg = C / G;
          const uint64_t woff = P.wreserve((uint64_t)OC * KH * KW * cg);
          for (int o = 0; o < OC; ++o)
            for (int c = 0; c < cg; ++c)
              for (int r = 0; r < KH; ++r)
                for (int s = 0; s < KW; ++s)
                  m->whost[woff + (((uint64_t)o * KH + r) * KW + s) * cg + c] = W.host[(((uint64_t)o * cg + c) * KH + r) * KW + s];
          uint64_t boff = ~0ull;
          if (B) {
            boff = P.wreserve(ocpad);
            for (int o = 0; o < OC; ++o) m->whost[boff + o] = B->host[o];
          }
          const int s = add_step(ni, OP_CONV, 4, fl, [=](StepRec& r) {
            const Buf* xbp = &m->bufs[xb];
            const Buf* ybp = &m->bufs[yb];
            const Buf* rbp = rb >= 0 ? &m->bufs[rb] : nullptr;
            r.run = [=](cudaStream_t st) {
              return launch_grouped_nhwc(xbp->ptr, m->wdev + woff, boff != ~0ull ? m->wdev + boff : nullptr,
                                         rbp ? rbp->ptr : nullptr, ybp->ptr, N, H, Wd, C, cpad, OH, OW, OC, ocpad, KH,
                                         KW, SH, SW, PH, PW, DH, DW, G, act, rnd, st);
            };
            return 0;
          });
          P.touch(xb, s);
          P.touch(yb, s);
          if (rb >= 0) P.touch(rb, s);
        }
        produced[yb] = 1;
        break;
      }
      case OP_MAXPOOL:
      case OP_AVGPOOL: {
        PoolParams pp{};
        if (nd.params.size() >= sizeof(PoolParams)) std::memcpy(&pp, nd.params.data(), sizeof(pp));
        const TensorRec& X = m->tensors[nd.in[0]];
        const TensorRec& Y = m->tensors[nd.out[0]];
        if (X.ndim != 4 || Y.ndim != 4) {
          set_error("plan: pool node %d needs 4-D tensors", ni);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        const int xb = ensure_nhwc(nd.in[0], ni);
        const int yb = nd.out[0];
        set_nhwc(m->bufs[yb], Y);
        const int KH = pp.kernel_shape[0] ? pp.kernel_shape[0] : 1, KW = pp.kernel_shape[1] ? pp.kernel_shape[1] : 1;
        const int SH = pp.strides[0] ? pp.strides[0] : 1, SW = pp.strides[1] ? pp.strides[1] : 1;
        const int PH = pp.pads[0], PW = pp.pads[1], cip = pp.count_include_pad;
        const bool is_max = nd.op == OP_MAXPOOL;
        const int s = add_step(ni, nd.op, 5, 0, [=](StepRec& r) {
          const Buf* x = &m->bufs[xb];
          const Buf* y = &m->bufs[yb];
          r.run = [=](cudaStream_t st) {
            return is_max ? launch_maxpool_nhwc(x->ptr, y->ptr, x->n, x->h, x->w, x->cpad, y->h, y->w, KH, KW, SH, SW,
                                                PH, PW, st)
                          : launch_avgpool_nhwc(x->ptr, y->ptr, x->n, x->h, x->w, x->cpad, y->h, y->w, KH, KW, SH, SW,
                                                PH, PW, cip, st);
          };
          return 0;
        });
        P.touch(xb, s);
        P.touch(yb, s);
        produced[yb] = 1;
        break;
      }
      case OP_GAP: {
        const TensorRec& Y = m->tensors[nd.out[0]];
        const int xb = ensure_nhwc(nd.in[0], ni);
        if (xb < 0) {
          set_error("plan: GlobalAveragePool node %d needs a 4-D input", ni);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        const int yb = nd.out[0];
        set_nhwc(m->bufs[yb], Y);  // [N, C, 1, 1] -> NHWC == [N][cpad]
        const int rnd = P.round_out;
        const int s = add_step(ni, nd.op, 5, 0, [=](StepRec& r) {
          const Buf* x = &m->bufs[xb];
          const Buf* y = &m->bufs[yb];
          r.run = [=](cudaStream_t st) {
            return launch_gap_nhwc(x->ptr, y->ptr, x->n, x->h * x->w, x->cpad, st, rnd);
          };
          return 0;
        });
        P.touch(xb, s);
        P.touch(yb, s);
        produced[yb] = 1;
        break;
      }
      case OP_FLATTEN:
      case OP_RESHAPE:
      case OP_IDENTITY: {
        const int xid = nd.in[0], yid = nd.out[0];
        const TensorRec& Y = m->tensors[yid];
        Buf& xbuf = m->bufs[xid];
        if (!(m->flags & SPINN_CUDA_PLAN_NO_FUSE) && xbuf.lay == LAY_NHWC &&
            reshape_feeds_gather(m, ni, readers, reader_node)) {
          // an NCHW view that only a last-axis Concat reads: it gathers from the NHWC tensor
          lazy_nchw[yid] = xid;
          set_row(m->bufs[yid], Y);
          m->bufs[yid].bytes = 0;
          produced[yid] = 1;
          break;
        }
        const bool nhwc_trivial = xbuf.lay == LAY_NHWC && xbuf.h * xbuf.w == 1 && xbuf.cpad == xbuf.c;
        int src = xid;
        if (xbuf.lay == LAY_NHWC && !nhwc_trivial) src = ensure_row(xid, ni);
        set_row(m->bufs[yid], Y);
        m->bufs[yid].alias = src;  // same bytes, row-major view
        const int s = add_step(ni, nd.op, 0, 0, [](StepRec& r) {
          r.run = [](cudaStream_t) { return 0; };
          return 0;
        });
        P.touch(src, s);
        produced[yid] = 1;
        break;
      }
      case OP_GEMM: {
        GemmParams gp{1.0f, 1.0f, 0, 0, {0, 0}};
        if (nd.params.size() >= sizeof(GemmParams)) std::memcpy(&gp, nd.params.data(), sizeof(gp));
        const TensorRec& A = m->tensors[nd.in[0]];
        const TensorRec& Bw = m->tensors[nd.in[1]];
        const TensorRec& Y = m->tensors[nd.out[0]];
        if (A.ndim != 2 || Bw.ndim != 2 || !Bw.host || A.is_weight) {
          set_error("plan: Gemm node %d: activation A and constant 2-D B required", ni);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        const int M = gp.transA ? A.dims[1] : A.dims[0];
        const int K = gp.transA ? A.dims[0] : A.dims[1];
        const int N = gp.transB ? Bw.dims[0] : Bw.dims[1];
        const int Np = round4(N), Kp = round4(K);
        const int kpad = tc_num_kb(K) * 32;
        const uint64_t woff = P.wreserve((uint64_t)Np * kpad);
        for (int n = 0; n < N; ++n)
          for (int k = 0; k < K; ++k)
            m->whost[woff + (uint64_t)n * kpad + k] =
                host_round_tf32(gp.transB ? Bw.host[(uint64_t)n * K + k] : Bw.host[(uint64_t)k * N + n]);
        uint64_t boff = ~0ull, roff = ~0ull;
        const TensorRec* Cb = nd.in.size() > 2 ? &m->tensors[nd.in[2]] : nullptr;
        if (Cb && Cb->host && gp.beta != 0.0f) {
          if (Cb->elems == (uint64_t)N) {
            boff = P.wreserve(Np);
            for (int n = 0; n < N; ++n) m->whost[boff + n] = gp.beta * Cb->host[n];
          } else if (Cb->elems == (uint64_t)M * N) {
            roff = P.wreserve((uint64_t)M * Np);
            for (int i = 0; i < M; ++i)
              for (int n = 0; n < N; ++n) m->whost[roff + (uint64_t)i * Np + n] = gp.beta * Cb->host[(uint64_t)i * N + n];
          } else {
            set_error("plan: Gemm node %d: C must be [N] or [M,N]", ni);
            return SPINN_CUDA_EUNSUPPORTED;
          }
        }
        if (gp.transA && Kp != K) {
          set_error("plan: Gemm node %d: transA with K=%d not a multiple of 4 is not supported", ni, K);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        int ab = ensure_row(nd.in[0], ni);
        // A operand: row-major [M][Kp]; transposed or misaligned inputs go through a temp
        int at = -1;
        if (gp.transA || Kp != K) {
          Buf tb;
          tb.lay = LAY_ROW;
          tb.bytes = (uint64_t)M * Kp * 4;
          at = P.new_buf(tb);
        }
        int yt = -1;
        const int yb = nd.out[0];
        set_row(m->bufs[yb], Y);
        if (Np != N) {
          Buf tb;
          tb.lay = LAY_ROW;
          tb.bytes = (uint64_t)M * Np * 4;
          yt = P.new_buf(tb);
        }
        const float alpha = gp.alpha;
        const int transA = gp.transA;
        const int s = add_step(ni, OP_GEMM, 2, 2.0 * M * N * K, [=](StepRec& r) {
          const Buf* a = &m->bufs[ab];
          const Buf* atp = at >= 0 ? &m->bufs[at] : nullptr;
          const Buf* y = &m->bufs[yb];
          const Buf* ytp = yt >= 0 ? &m->bufs[yt] : nullptr;
          TcGemmArgs q;
          q.a_mode = 1;
          q.M = M;
          q.K = K;
          q.lda = Kp;
          q.kpad = kpad;
          q.N = Np;
          q.ldy = Np;
          note_ws(m, q);
          r.run = [=](cudaStream_t st) {
            const float* A_ = a->ptr;
            if (atp) {
              if (transA) {
                int rc = launch_transpose(a->ptr, atp->ptr, 1, K, M, st);
                if (rc) return rc;
              } else {
                SPINN_CUDA_TRY(cudaMemcpy2DAsync(atp->ptr, (size_t)Kp * 4, a->ptr, (size_t)K * 4, (size_t)K * 4, M,
                                                 cudaMemcpyDeviceToDevice, st));
              }
              A_ = atp->ptr;
            }
            TcGemmArgs g;
            g.a_mode = 1;
            g.x = A_;
            g.M = M;
            g.K = K;
            g.lda = Kp;
            g.wt = m->wdev + woff;
            g.kpad = kpad;
            g.N = Np;
            g.bias = boff != ~0ull ? m->wdev + boff : nullptr;
            g.res = roff != ~0ull ? m->wdev + roff : nullptr;
            g.ldr = Np;
            g.y = ytp ? ytp->ptr : y->ptr;
            g.ldy = Np;
            g.alpha = alpha;
            g.ws = m->splitk_ws;
            g.ws_bytes = m->splitk_bytes;
            int rc = tc_gemm_launch(g, st);
            if (rc) return rc;
            if (ytp)
              SPINN_CUDA_TRY(cudaMemcpy2DAsync(y->ptr, (size_t)N * 4, ytp->ptr, (size_t)Np * 4, (size_t)N * 4, M,
                                               cudaMemcpyDeviceToDevice, st));
            return 0;
          };
          return 0;
        });
        P.touch(ab, s);
        P.touch(yb, s);
        if (at >= 0) P.touch(at, s);
        if (yt >= 0) P.touch(yt, s);
        produced[yb] = 1;
        break;
      }
      case OP_ADD:
      case OP_MUL:
      case OP_SUB:
      case OP_DIV: {
        const int aid = nd.in[0], bid = nd.in[1], yid = nd.out[0];
        const TensorRec& Ta = m->tensors[aid];
        const TensorRec& Tb = m->tensors[bid];
        const TensorRec& Ty = m->tensors[yid];
        const int op = nd.op == OP_ADD ? ELT_ADD : nd.op == OP_MUL ? ELT_MUL : nd.op == OP_SUB ? ELT_SUB : ELT_DIV;
        // fast path: both operands activations of the output's shape, same NHWC layout
        const bool same = !Ta.is_weight && !Tb.is_weight && Ta.elems == Ty.elems && Tb.elems == Ty.elems &&
                          m->bufs[aid].lay == LAY_NHWC && m->bufs[bid].lay == LAY_NHWC && op != ELT_DIV;
        int ab, bb;
        uint64_t wa = ~0ull, wb = ~0ull;
        if (same) {
          ab = aid;
          bb = bid;
          set_nhwc(m->bufs[yid], Ty);
        } else {
          if (Ta.is_weight) {
            wa = P.wreserve(Ta.elems);
            std::memcpy(&m->whost[wa], Ta.host, Ta.elems * 4);
            ab = -1;
          } else {
            ab = ensure_row(aid, ni);
          }
          if (Tb.is_weight) {
            wb = P.wreserve(Tb.elems);
            std::memcpy(&m->whost[wb], Tb.host, Tb.elems * 4);
            bb = -1;
          } else {
            bb = ensure_row(bid, ni);
          }
          set_row(m->bufs[yid], Ty);
        }
        const long na = (long)Ta.elems, nbv = (long)Tb.elems;
        const int s = add_step(ni, nd.op, 6, 0, [=](StepRec& r) {
          const Buf* a = ab >= 0 ? &m->bufs[ab] : nullptr;
          const Buf* b = bb >= 0 ? &m->bufs[bb] : nullptr;
          const Buf* y = &m->bufs[yid];
          r.run = [=](cudaStream_t st) {
            const float* pa = a ? a->ptr : m->wdev + wa;
            const float* pb = b ? b->ptr : m->wdev + wb;
            if (same) {
              const long n = (long)y->bytes / 4;
              return launch_binary(pa, n, pb, n, y->ptr, n, op, 0, st);
            }
            return launch_binary(pa, na, pb, nbv, y->ptr, (long)(y->bytes / 4), op, 0, st);
          };
          return 0;
        });
        if (ab >= 0) P.touch(ab, s);
        if (bb >= 0) P.touch(bb, s);
        P.touch(yid, s);
        produced[yid] = 1;
        break;
      }
      case OP_RELU:
      case OP_SIGMOID: {
        const int xid = nd.in[0], yid = nd.out[0];
        Buf& xb = m->bufs[xid];
        if (xb.lay == LAY_NHWC)
          set_nhwc(m->bufs[yid], m->tensors[yid]);
        else
          set_row(m->bufs[yid], m->tensors[yid]);
        const int op = nd.op == OP_RELU ? UN_RELU : UN_SIGMOID;
        // Sigmoid of a zero pad channel is 0.5: row layout keeps no pad channels.
        int src = xid;
        if (op == UN_SIGMOID && xb.lay == LAY_NHWC && xb.cpad != xb.c) {
          src = ensure_row(xid, ni);
          set_row(m->bufs[yid], m->tensors[yid]);
        }
        const int s = add_step(ni, nd.op, 6, 0, [=](StepRec& r) {
          const Buf* x = &m->bufs[src];
          const Buf* y = &m->bufs[yid];
          r.run = [=](cudaStream_t st) { return launch_unary(x->ptr, y->ptr, (long)(y->bytes / 4), op, st); };
          return 0;
        });
        P.touch(src, s);
        P.touch(yid, s);
        produced[yid] = 1;
        break;
      }
      case OP_BN: {
        // standalone BatchNormalization (op_batch_norm, SPINN/run_time/ops/norm/batch_norm.c:17-76)
        BnParams bp{1e-5f, 0.9f, 0, {0, 0, 0}};
        if (nd.params.size() >= sizeof(BnParams)) std::memcpy(&bp, nd.params.data(), sizeof(bp));
        if (nd.in.size() < 5) {
          set_error("plan: BatchNormalization node %d needs 5 inputs", ni);
          return SPINN_CUDA_EFORMAT;
        }
        const TensorRec &g = m->tensors[nd.in[1]], &b = m->tensors[nd.in[2]], &mu = m->tensors[nd.in[3]],
                        &var = m->tensors[nd.in[4]];
        if (!g.host || !b.host || !mu.host || !var.host) {
          set_error("plan: BatchNormalization node %d needs constant statistics", ni);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        const int xb = ensure_nhwc(nd.in[0], ni);
        if (xb < 0) {
          set_error("plan: BatchNormalization node %d needs a 4-D input", ni);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        const int yid = nd.out[0];
        set_nhwc(m->bufs[yid], m->tensors[yid]);
        const int C = m->bufs[yid].c, cpad = m->bufs[yid].cpad;
        const uint64_t so = P.wreserve(cpad), ho = P.wreserve(cpad);
        for (int c = 0; c < C; ++c) {
          const float a = g.host[c] / std::sqrt(var.host[c] + bp.epsilon);
          m->whost[so + c] = a;
          m->whost[ho + c] = b.host[c] - mu.host[c] * a;
        }
        const int s = add_step(ni, nd.op, 6, 0, [=](StepRec& r) {
          const Buf* x = &m->bufs[xb];
          const Buf* y = &m->bufs[yid];
          r.run = [=](cudaStream_t st) {
            return launch_channel_affine_nhwc(x->ptr, y->ptr, (long)y->n * y->h * y->w, y->cpad, m->wdev + so,
                                              m->wdev + ho, st);
          };
          return 0;
        });
        P.touch(xb, s);
        P.touch(yid, s);
        produced[yid] = 1;
        break;
      }
      case OP_CONCAT:
      case OP_SPLIT: {
        // Concat (SPINN/run_time/ops/tensor/concat.c) / Split (tensor/split.c) as strided 2-D
        // copies: along the channel axis of NHWC tensors, or along any axis of row-major ones.
        const bool is_cat = nd.op == OP_CONCAT;
        int axis = is_cat ? 1 : 0;
        if (nd.params.size() >= 4) std::memcpy(&axis, nd.params.data(), 4);
        const std::vector<uint16_t>& parts = is_cat ? nd.in : nd.out;
        const int whole = is_cat ? nd.out[0] : nd.in[0];
        const TensorRec& TW = m->tensors[whole];
        if (axis < 0) axis += TW.ndim;
        if (axis < 0 || axis >= TW.ndim) {
          set_error("plan: %s node %d axis out of range", is_cat ? "Concat" : "Split", ni);
          return SPINN_CUDA_EFORMAT;
        }
        for (auto id : parts)
          if (m->tensors[id].is_weight) {
            set_error("plan: Concat/Split node %d with constant operands", ni);
            return SPINN_CUDA_EUNSUPPORTED;
          }
        const bool nhwc = TW.ndim == 4 && axis == 1;
        if (!(m->flags & SPINN_CUDA_PLAN_NO_FUSE) && is_cat && nhwc && parts.size() >= 2 && parts.size() <= 4 &&
            readers[whole] == 1 && reader_node[whole] > ni && m->nodes[reader_node[whole]].in[0] == whole &&
            reshape_feeds_gather(m, reader_node[whole], readers, reader_node)) {
          // a channel Concat viewed as NCHW by a Reshape that a last-axis Concat gathers: that
          // gather reads each part where it lies
          std::vector<int> pbv;
          for (auto id : parts) pbv.push_back(ensure_nhwc(id, ni));
          bool all = true;
          for (int b : pbv) all &= b >= 0;
          if (all) {
            virt_cat[whole] = pbv;
            set_nhwc(m->bufs[whole], TW);
            m->bufs[whole].bytes = 0;
            produced[whole] = 1;
            break;
          }
        }
        if (is_cat && TW.ndim == 3 && axis == 2) {
          bool any_lazy = false;
          for (auto id : parts) any_lazy |= lazy_nchw.count(id) > 0;
          if (any_lazy) {
            // last-axis Concat of [N][C][L_i] parts, some of them NCHW views of NHWC tensors (or
            // of channel Concats of them): one gathering pass writes the result
            struct Piece {
              int buf, nhwc, ld, chans, len, dst_c, dst_l;
            };
            std::vector<Piece> pcs;
            const int N = TW.dims[0], C = TW.dims[1];
            int col = 0;
            for (auto id : parts) {
              const TensorRec& T = m->tensors[id];
              if (T.ndim != 3 || (int)T.dims[0] != N || (int)T.dims[1] != C) {
                set_error("plan: Concat node %d: parts differ outside the concatenated axis", ni);
                return SPINN_CUDA_EFORMAT;
              }
              const int L = T.dims[2];
              auto lz = lazy_nchw.find(id);
              if (lz != lazy_nchw.end()) {
                auto vc = virt_cat.find(lz->second);
                if (vc != virt_cat.end()) {
                  int cc = 0;
                  for (int pb : vc->second) {
                    pcs.push_back({pb, 1, m->bufs[pb].cpad, m->bufs[pb].c, L, cc, col});
                    cc += m->bufs[pb].c;
                  }
                } else {
                  const int src = lz->second;
                  pcs.push_back({src, 1, m->bufs[src].cpad, C, L, 0, col});
                }
              } else {
                pcs.push_back({ensure_row(id, ni), 0, L, C, L, 0, col});
              }
              col += L;
            }
            if ((int)pcs.size() > kGatherMaxPieces) {
              set_error("plan: Concat node %d gathers %d pieces (at most %d)", ni, (int)pcs.size(),
                        kGatherMaxPieces);
              return SPINN_CUDA_EUNSUPPORTED;
            }
            set_row(m->bufs[whole], TW);
            const int L = TW.dims[2];
            const int s = add_step(ni, nd.op, 6, 0, [=](StepRec& r) {
              const Buf* w = &m->bufs[whole];
              std::vector<const Buf*> src;
              for (const Piece& p : pcs) src.push_back(&m->bufs[p.buf]);
              r.run = [=](cudaStream_t st) {
                GatherPieces g{};
                g.n = (int)pcs.size();
                for (size_t k = 0; k < pcs.size(); ++k) {
                  g.src[k] = src[k]->ptr;
                  g.nhwc[k] = pcs[k].nhwc;
                  g.ld[k] = pcs[k].ld;
                  g.c0[k] = 0;
                  g.chans[k] = pcs[k].chans;
                  g.len[k] = pcs[k].len;
                  g.dst_c[k] = pcs[k].dst_c;
                  g.dst_l[k] = pcs[k].dst_l;
                }
                return launch_gather_rows(g, w->ptr, N, C, L, st);
              };
              return 0;
            });
            P.touch(whole, s);
            for (const Piece& p : pcs) P.touch(p.buf, s);
            produced[whole] = 1;
            break;
          }
        }
        if (!(m->flags & SPINN_CUDA_PLAN_NO_FUSE) && is_cat && nhwc && parts.size() >= 2 && parts.size() <= 4 &&
            readers[whole] == 1 &&
            reader_node[whole] > ni && concat_feeds_tc_conv(m, reader_node[whole], whole, parts)) {
          // the convolution reading this Concat fetches each channel block from its part
          std::vector<int> pbv;
          for (auto id : parts) pbv.push_back(ensure_nhwc(id, ni));
          bool all = true;
          for (int b : pbv) all &= b >= 0;
          if (all) {
            virt_cat[whole] = pbv;
            set_nhwc(m->bufs[whole], TW);
            m->bufs[whole].bytes = 0;  // no storage of its own
            produced[whole] = 1;
            break;
          }
        }
        std::vector<int> pb;  // buffers of the parts
        int wb;
        if (nhwc) {
          if (is_cat) {
            for (auto id : parts) pb.push_back(ensure_nhwc(id, ni));
            wb = whole;
            set_nhwc(m->bufs[wb], TW);
          } else {
            wb = ensure_nhwc(whole, ni);
            for (auto id : parts) {
              set_nhwc(m->bufs[id], m->tensors[id]);
              pb.push_back(id);
            }
          }
        } else {
          if (is_cat) {
            for (auto id : parts) pb.push_back(ensure_row(id, ni));
            wb = whole;
            set_row(m->bufs[wb], TW);
          } else {
            wb = ensure_row(whole, ni);
            for (auto id : parts) {
              set_row(m->bufs[id], m->tensors[id]);
              pb.push_back(id);
            }
          }
        }
        long outer = 1, inner = 1;
        for (int d = 0; d < axis; ++d) outer *= TW.dims[d];
        for (int d = axis + 1; d < TW.ndim; ++d) inner *= TW.dims[d];
        std::vector<int> sizes;
        for (auto id : parts) sizes.push_back((int)m->tensors[id].dims[axis]);
        const int s = add_step(ni, nd.op, 6, 0, [=](StepRec& r) {
          std::vector<const Buf*> pp;
          for (int b : pb) pp.push_back(&m->bufs[b]);
          const Buf* w = &m->bufs[wb];
          r.run = [=](cudaStream_t st) -> int {
            // one row-strided copy kernel per part; NHWC pad lanes of every destination are
            // written as zeros by the copy that owns them
            int off = 0;
            const long rows = nhwc ? (long)w->n * w->h * w->w : outer;
            const int wld = nhwc ? w->cpad : (int)(w->bytes / 4 / outer);
            if (is_cat && (int)pp.size() <= kCatMaxParts && wld % 4 == 0) {
              // float4-aligned parts: the whole destination row in one launch
              CatParts cp{};
              cp.n = (int)pp.size();
              bool ok = true;
              for (size_t i = 0; i < pp.size(); ++i) {
                const int width = nhwc ? sizes[i] : (int)(sizes[i] * inner);
                cp.src[i] = pp[i]->ptr;
                cp.ld[i] = nhwc ? pp[i]->cpad : width;
                cp.off[i] = off;
                cp.width[i] = width;
                ok &= width % 4 == 0 && off % 4 == 0 && cp.ld[i] % 4 == 0;
                off += width;
              }
              if (ok) return launch_concat_rows(cp, w->ptr, wld, rows, wld, st);
              off = 0;
            }
            if (!is_cat && (int)pp.size() <= kCatMaxParts && wld % 4 == 0) {
              // dense float4-aligned parts (no pad lanes to zero): one launch
              SplitParts sp{};
              sp.n = (int)pp.size();
              bool ok = true;
              for (size_t i = 0; i < pp.size(); ++i) {
                const int width = nhwc ? sizes[i] : (int)(sizes[i] * inner);
                const int pld = nhwc ? pp[i]->cpad : width;
                sp.dst[i] = pp[i]->ptr;
                sp.ld[i] = pld;
                sp.off[i] = off;
                sp.width[i] = width;
                ok &= width % 4 == 0 && pld == width;
                off += width;
              }
              if (ok) return launch_split_rows(sp, w->ptr, wld, rows, st);
              off = 0;
            }
            for (size_t i = 0; i < pp.size(); ++i) {
              const Buf* p = pp[i];
              const int width = nhwc ? sizes[i] : (int)(sizes[i] * inner);
              const int pld = nhwc ? p->cpad : width;
              int rc;
              if (is_cat) {
                const int fill = (nhwc && i + 1 == pp.size()) ? wld - off : width;
                rc = launch_copy_rows(p->ptr, pld, w->ptr + off, wld, rows, width, fill, st);
              } else {
                rc = launch_copy_rows(w->ptr + off, wld, p->ptr, pld, rows, width, pld, st);
              }
              if (rc) return rc;
              off += width;
            }
            return 0;
          };
          return 0;
        });
        P.touch(wb, s);
        for (int b : pb) P.touch(b, s);
        for (auto id : nd.out) produced[id] = 1;
        break;
      }
      case OP_RESIZE: {
        const TensorRec& X = m->tensors[nd.in[0]];
        const TensorRec& Y = m->tensors[nd.out[0]];
        if (X.ndim != 4 || Y.ndim != 4 || X.dims[0] != Y.dims[0] || X.dims[1] != Y.dims[1]) {
          set_error("plan: Resize node %d: only 4-D spatial nearest resize is supported", ni);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        const int xb = ensure_nhwc(nd.in[0], ni);
        const int yb = nd.out[0];
        set_nhwc(m->bufs[yb], Y);
        const int s = add_step(ni, nd.op, 5, 0, [=](StepRec& r) {
          const Buf* x = &m->bufs[xb];
          const Buf* y = &m->bufs[yb];
          r.run = [=](cudaStream_t st) {
            return launch_resize_nearest_nhwc(x->ptr, y->ptr, x->n, x->h, x->w, x->cpad, y->h, y->w, st);
          };
          return 0;
        });
        P.touch(xb, s);
        P.touch(yb, s);
        produced[yb] = 1;
        break;
      }
      case OP_TRANSPOSE: {
        const TensorRec& X = m->tensors[nd.in[0]];
        uint8_t perm[8];
        for (int d = 0; d < X.ndim; ++d) perm[d] = (uint8_t)(X.ndim - 1 - d);  // default: reverse
        if (nd.params.size() >= 9 && nd.params[8] == X.ndim)
          for (int d = 0; d < X.ndim; ++d) perm[d] = nd.params[d];
        // a swap of the last two axes (leading axes in place) is a batch of matrix transposes
        bool last2 = X.ndim >= 2 && perm[X.ndim - 2] == X.ndim - 1 && perm[X.ndim - 1] == X.ndim - 2;
        for (int d = 0; d + 2 < X.ndim; ++d) last2 &= perm[d] == d;
        const int yb = nd.out[0];
        if (last2 && !(m->flags & SPINN_CUDA_PLAN_NO_FUSE) && readers[yb] == 1 && reader_node[yb] > ni &&
            m->nodes[reader_node[yb]].op == OP_MATMUL && m->nodes[reader_node[yb]].in.size() >= 2 &&
            m->nodes[reader_node[yb]].in[1] == yb && m->nodes[reader_node[yb]].in[0] != yb && X.dtype != kDtypeInt64) {
          // B of the MatMul that reads it: the MatMul packs B from its transpose anyway, which is
          // this tensor's input
          b_trans[yb] = nd.in[0];
          set_row(m->bufs[yb], m->tensors[yb]);
          m->bufs[yb].bytes = 0;
          produced[yb] = 1;
          break;
        }
        const int xb = ensure_row(nd.in[0], ni);
        set_row(m->bufs[yb], m->tensors[yb]);
        std::vector<uint32_t> dims(X.dims, X.dims + 8);
        std::vector<uint8_t> pv(perm, perm + 8);
        const int ndim = X.ndim;
        long mats = 1;
        for (int d = 0; d + 2 < ndim; ++d) mats *= X.dims[d];
        const int rows = ndim >= 2 ? (int)X.dims[ndim - 2] : 1, cols = ndim >= 1 ? (int)X.dims[ndim - 1] : 1;
        const int s = add_step(ni, nd.op, 7, 0, [=](StepRec& r) {
          const Buf* x = &m->bufs[xb];
          const Buf* y = &m->bufs[yb];
          r.run = [=](cudaStream_t st) -> int {
            if (!last2) return launch_permute(x->ptr, y->ptr, ndim, dims.data(), pv.data(), st);
            const size_t plane = (size_t)rows * cols;
            if (plane == 0) return 0;
            for (long b0 = 0; b0 < mats; b0 += 65535) {  // grid.z holds at most 65535 matrices
              const int nb = (int)std::min<long>(65535, mats - b0);
              const int rc = launch_transpose(x->ptr + b0 * plane, y->ptr + b0 * plane, nb, rows, cols, st);
              if (rc) return rc;
            }
            return 0;
          };
          return 0;
        });
        P.touch(xb, s);
        P.touch(yb, s);
        produced[yb] = 1;
        break;
      }
      case OP_TOPK: {
        // TopK (SPINN/run_time/ops/tensor/topk.c): last axis, k largest, sorted descending,
        // as the reference (which ignores the axis/largest/sorted attributes).
        if (nd.in.size() < 2 || nd.out.size() < 2) {
          set_error("plan: TopK node %d needs inputs X, K and outputs values, indices", ni);
          return SPINN_CUDA_EFORMAT;
        }
        const TensorRec& X = m->tensors[nd.in[0]];
        const TensorRec& Kt = m->tensors[nd.in[1]];
        if (!Kt.is_weight || !Kt.host || Kt.elems < 1) {
          set_error("plan: TopK node %d: K must be a constant", ni);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        int64_t kv = 0;
        if (Kt.dtype == kDtypeInt64)
          std::memcpy(&kv, Kt.host, 8);
        else
          kv = (int64_t)Kt.host[0];
        const int n = X.ndim ? (int)X.dims[X.ndim - 1] : 1;
        if (n < 1 || n > kTopkMaxN) {
          set_error("plan: TopK node %d: last axis %d outside [1, %d]", ni, n, kTopkMaxN);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        const int k = (int)std::max<int64_t>(0, std::min<int64_t>(kv, n));
        const long rows = (long)(X.elems / n);
        const TensorRec& V = m->tensors[nd.out[0]];
        const TensorRec& I = m->tensors[nd.out[1]];
        if (V.elems != (uint64_t)rows * k || I.elems != (uint64_t)rows * k || I.dtype != kDtypeInt64) {
          set_error("plan: TopK node %d: outputs must be [rows, %d] float and int64", ni, k);
          return SPINN_CUDA_EFORMAT;
        }
        const int xb = ensure_row(nd.in[0], ni);
        const int vb = nd.out[0], ib = nd.out[1];
        set_row(m->bufs[vb], V);
        set_row(m->bufs[ib], I);
        const int s = add_step(ni, nd.op, 6, 0, [=](StepRec& r) {
          const Buf* x = &m->bufs[xb];
          const Buf* v = &m->bufs[vb];
          const Buf* ix = &m->bufs[ib];
          r.run = [=](cudaStream_t st) {
            return launch_topk(x->ptr, rows, n, k, v->ptr, reinterpret_cast<int64_t*>(ix->ptr), st);
          };
          return 0;
        });
        P.touch(xb, s);
        P.touch(vb, s);
        P.touch(ib, s);
        produced[vb] = 1;
        produced[ib] = 1;
        break;
      }
      case OP_SOFTMAX: {
        const TensorRec& X = m->tensors[nd.in[0]];
        int axis = -1;
        if (nd.params.size() >= 4) std::memcpy(&axis, nd.params.data(), 4);
        if (axis < 0) axis += X.ndim;
        if (axis < 0 || axis >= X.ndim) {
          set_error("plan: Softmax node %d axis out of range", ni);
          return SPINN_CUDA_EFORMAT;
        }
        long outer = 1, inner = 1;
        for (int d = 0; d < axis; ++d) outer *= X.dims[d];
        for (int d = axis + 1; d < X.ndim; ++d) inner *= X.dims[d];
        const int dim = X.dims[axis];
        const int xb = ensure_row(nd.in[0], ni);
        const int yb = nd.out[0];
        set_row(m->bufs[yb], m->tensors[yb]);
        const int s = add_step(ni, nd.op, 6, 0, [=](StepRec& r) {
          const Buf* x = &m->bufs[xb];
          const Buf* y = &m->bufs[yb];
          r.run = [=](cudaStream_t st) { return launch_softmax(x->ptr, y->ptr, outer, dim, inner, st); };
          return 0;
        });
        P.touch(xb, s);
        P.touch(yb, s);
        produced[yb] = 1;
        break;
      }
      case OP_MATMUL: {
        // MatMul (SPINN/run_time/ops/mm/matmul.c) with ONNX broadcasting of a 2-D B: per batch a
        // tcgen05 GEMM in split-tf32 (A' = [A_hi|A_lo|A_hi], B' = [B_hi|B_hi|B_lo] along K), so
        // activation x activation products (attention scores feeding a softmax) keep about
        // fp32 accuracy; these GEMMs are small next to the convolutions.
        const TensorRec& A = m->tensors[nd.in[0]];
        const TensorRec& Bt = m->tensors[nd.in[1]];
        const TensorRec& Y = m->tensors[nd.out[0]];
        if (A.is_weight || A.ndim < 2 || Bt.ndim < 2) {
          set_error("plan: MatMul node %d needs an activation A and 2-D+ operands", ni);
          return SPINN_CUDA_EUNSUPPORTED;
        }
        const int M = A.dims[A.ndim - 2], K = A.dims[A.ndim - 1];
        const int K2 = Bt.dims[Bt.ndim - 2], N = Bt.dims[Bt.ndim - 1];
        long batch = 1, batch_b = 1;
        for (int d = 0; d < A.ndim - 2; ++d) batch *= A.dims[d];
        for (int d = 0; d < Bt.ndim - 2; ++d) batch_b *= Bt.dims[d];
        if (K != K2 || (batch_b != 1 && batch_b != batch)) {
          set_error("plan: MatMul node %d shapes do not match", ni);
          return SPINN_CUDA_EFORMAT;
        }
        const int seg = round4(K), Np = round4(N), kpad = tc_num_kb(3 * seg) * 32;
        const int ab = ensure_row(nd.in[0], ni);
        Buf t;
        t.lay = LAY_ROW;
        t.bytes = (uint64_t)batch * M * 3 * seg * 4;
        const int at = P.new_buf(t);  // A' split-packed
        uint64_t woff = ~0ull;
        int bb = -1, btt = -1, bpt = -1;
        if (Bt.is_weight) {
          woff = P.wreserve((uint64_t)batch_b * Np * kpad);
          for (long bi = 0; bi < batch_b; ++bi)
            for (int n = 0; n < N; ++n)
              for (int k = 0; k < K; ++k) {
                const float v = Bt.host[((uint64_t)bi * K + k) * N + n];
                const float hi = host_round_tf32(v), lo = host_round_tf32(v - hi);
                float* row = &m->whost[woff + ((uint64_t)bi * Np + n) * kpad];
                row[k] = hi;
                row[seg + k] = hi;
                row[2 * seg + k] = lo;
              }
        } else {
          auto bt_it = b_trans.find(nd.in[1]);
          if (bt_it != b_trans.end()) {
            // B is the transpose of a [.., N, K] tensor: that tensor is B's [N][K] form already
            btt = ensure_row(bt_it->second, ni);
          } else {
            bb = ensure_row(nd.in[1], ni);
            t.bytes = (uint64_t)batch_b * N * K * 4;
            btt = P.new_buf(t);
          }
          t.bytes = (uint64_t)batch_b * Np * kpad * 4;
          bpt = P.new_buf(t);
        }
        const int yb = nd.out[0];
        set_row(m->bufs[yb], Y);
        int yt = -1;
        if (Np != N) {
          t.bytes = (uint64_t)batch * M * Np * 4;
          yt = P.new_buf(t);
        }
        const int s = add_step(ni, nd.op, 2, 2.0 * batch * M * N * K, [=](StepRec& r) {
          const Buf* a = &m->bufs[ab];
          const Buf* ap = &m->bufs[at];
          const Buf* b = bb >= 0 ? &m->bufs[bb] : nullptr;
          const Buf* bt = btt >= 0 ? &m->bufs[btt] : nullptr;
          const Buf* bp = bpt >= 0 ? &m->bufs[bpt] : nullptr;
          const Buf* y = &m->bufs[yb];
          const Buf* ytp = yt >= 0 ? &m->bufs[yt] : nullptr;
          TcGemmArgs q;
          q.a_mode = 1;
          q.M = M;
          q.K = 3 * seg;
          q.lda = 3 * seg;
          q.kpad = kpad;
          q.N = Np;
          q.ldy = Np;
          q.batch = (int)batch;
          q.b_batched = batch_b > 1;
          note_ws(m, q);
          r.run = [=](cudaStream_t st) -> int {
            if (seg != K) SPINN_CUDA_TRY(cudaMemsetAsync(ap->ptr, 0, ap->bytes, st));
            int rc = launch_split_tf32(a->ptr, ap->ptr, batch * M, K, K, seg, 3 * seg, 0, 1, 0, st);
            if (rc) return rc;
            const float* wbase = woff != ~0ull ? m->wdev + woff : nullptr;
            if (bt) {
              if (b) {
                rc = launch_transpose(b->ptr, bt->ptr, (int)batch_b, K, N, st);  // -> [batch_b][N][K]
                if (rc) return rc;
              }
              // zeros where the packing writes nothing: with seg == K only the K padding past
              // the three segments and the rows past N (a full clear would write the whole,
              // three times widened B once more)
              if (seg != K) {
                SPINN_CUDA_TRY(cudaMemsetAsync(bp->ptr, 0, bp->bytes, st));
              } else {
                if (kpad > 3 * seg)
                  SPINN_CUDA_TRY(cudaMemset2DAsync(bp->ptr + 3 * seg, (size_t)kpad * 4, 0, (size_t)(kpad - 3 * seg) * 4,
                                                   (size_t)batch_b * Np, st));
                if (Np > N)
                  SPINN_CUDA_TRY(cudaMemset2DAsync(bp->ptr + (size_t)N * kpad, (size_t)Np * kpad * 4, 0,
                                                   (size_t)(Np - N) * kpad * 4, (size_t)batch_b, st));
              }
              if (Np == N) {  // the planes are contiguous rows: one packing pass
                rc = launch_split_tf32(bt->ptr, bp->ptr, batch_b * N, K, K, seg, kpad, 0, 0, 1, st);
                if (rc) return rc;
              } else {
                for (long bi = 0; bi < batch_b; ++bi) {
                  rc = launch_split_tf32(bt->ptr + (size_t)bi * N * K, bp->ptr + (size_t)bi * Np * kpad, N, K, K, seg,
                                         kpad, 0, 0, 1, st);
                  if (rc) return rc;
                }
              }
              wbase = bp->ptr;
            }
            // every batch in one launch: A', Y (and B') planes back to back
            TcGemmArgs g;
            g.a_mode = 1;
            g.x = ap->ptr;
            g.M = M;
            g.K = 3 * seg;
            g.lda = 3 * seg;
            g.wt = wbase;
            g.kpad = kpad;
            g.N = Np;
            g.y = ytp ? ytp->ptr : y->ptr;
            g.ldy = Np;
            g.batch = (int)batch;
            g.b_batched = batch_b > 1;
            g.ws = m->splitk_ws;
            g.ws_bytes = m->splitk_bytes;
            rc = tc_gemm_launch(g, st);
            if (rc) return rc;
            if (ytp) return launch_copy_rows(ytp->ptr, Np, y->ptr, N, batch * M, N, N, st);
            return 0;
          };
          return 0;
        });
        P.touch(ab, s);
        P.touch(at, s);
        if (bb >= 0) P.touch(bb, s);
        if (btt >= 0) {
          P.touch(btt, s);
          P.touch(bpt, s);
        }
        if (yt >= 0) P.touch(yt, s);
        P.touch(yb, s);
        produced[yb] = 1;
        break;
      }
      default:
        set_error("plan: operator %d (node %d) has no device implementation", nd.op, ni);
        return SPINN_CUDA_EUNSUPPORTED;
    }
  }

  // graph outputs: NCHW / row-major staging outside the arena
  for (size_t i = 0; i < m->outputs.size(); ++i) {
    const int id = m->outputs[i];
    if (!produced[id]) {
      set_error("plan: graph output %d is never produced", id);
      return SPINN_CUDA_EFORMAT;
    }
    const TensorRec& t = m->tensors[id];
    const int src = P.root(id);
    const bool nhwc = m->bufs[id].lay == LAY_NHWC;
    const uint64_t obytes = t.elems * elem_bytes(t);
    // A row-major output that fills its own buffer is handed to the host where it lies: the
    // buffer leaves the arena (nothing reuses it), and no staging copy runs.
    bool direct = !nhwc && m->bufs[id].lay == LAY_ROW && m->bufs[src].lay == LAY_ROW && !m->bufs[src].external &&
                  m->bufs[src].bytes == obytes && obytes > 0;
    for (int ob : m->out_buf) direct &= ob != src;
    if (direct) {
      m->bufs[src].external = 1;
      m->out_buf.push_back(src);
      continue;
    }
    Buf st;
    st.lay = LAY_ROW;
    st.bytes = obytes;
    st.external = 1;
    const int sb = P.new_buf(st);
    m->out_buf.push_back(sb);
    const int s = add_step(-1, 0, 7, 0, [m, id, sb, nhwc](StepRec& r) {
      const Buf* x = &m->bufs[id];
      const Buf* xr = x;
      while (xr->alias >= 0) xr = &m->bufs[xr->alias];
      const Buf* y = &m->bufs[sb];
      r.run = [x, xr, y, nhwc](cudaStream_t st) -> int {
        if (nhwc) return launch_nhwc_to_nchw(xr->ptr, y->ptr, x->n, x->c, x->h, x->w, x->cpad, st);
        SPINN_CUDA_TRY(cudaMemcpyAsync(y->ptr, xr->ptr, y->bytes, cudaMemcpyDeviceToDevice, st));
        return 0;
      };
      return 0;
    });
    P.touch(src, s);
  }

  m->virt_cat = virt_cat;
  m->lazy_nchw = lazy_nchw;
  m->b_trans = b_trans;
  // arena
  const int nsteps = (int)m->steps.size();
  int rc = plan_arena(m, nsteps, budget);
  if (rc) return rc;
  if (m->arena_bytes) SPINN_CUDA_TRY(cudaMalloc(&m->arena, m->arena_bytes));
  for (auto& b : m->bufs) {
    if (b.alias >= 0) continue;
    if (b.external) {
      if (b.bytes) SPINN_CUDA_TRY(cudaMalloc(&b.ptr, align_up(b.bytes, 256)));
    } else if (b.offset >= 0) {
      b.ptr = reinterpret_cast<float*>(m->arena + b.offset);
    }
  }
  for (auto& b : m->bufs) {
    if (b.alias < 0) continue;
    int r = b.alias;
    while (m->bufs[r].alias >= 0) r = m->bufs[r].alias;
    b.ptr = m->bufs[r].ptr;
  }
  // weights
  m->wbytes = m->whost.size() * 4;
  if (m->wbytes) {
    SPINN_CUDA_TRY(cudaMalloc(&m->wdev, m->wbytes));
    SPINN_CUDA_TRY(cudaMemcpy(m->wdev, m->whost.data(), m->wbytes, cudaMemcpyHostToDevice));
  }
  std::vector<float>().swap(m->whost);
  // closures
  m->kernels = 0;
  for (int i = 0; i < nsteps; ++i) {
    rc = builders[i](m->steps[i]);
    if (rc) return rc;
    if (m->steps[i].kind != 0) ++m->kernels;
  }
  if (m->splitk_bytes) SPINN_CUDA_TRY(cudaMalloc(&m->splitk_ws, m->splitk_bytes));
  if (m->sk_used && m->splitk_bytes) {
    SPINN_CUDA_TRY(cudaMalloc(&m->sk_flags, kTcSkFlags * sizeof(int)));
    SPINN_CUDA_TRY(cudaMemset(m->sk_flags, 0, kTcSkFlags * sizeof(int)));
  }
  return 0;
}

// Device error check after a run.  A run that timed out may have left stream-K flags raised;
// they are cleared so that the model stays usable.
static int check_run(SpinnCudaModel* m, cudaStream_t st) {
  const int rc = check_device_error_flag(m->device, st);
  if (rc && m->sk_flags) {
    cudaMemsetAsync(m->sk_flags, 0, kTcSkFlags * sizeof(int), st);
    cudaStreamSynchronize(st);
  }
  return rc;
}

static int run_steps(SpinnCudaModel* m, cudaStream_t st, bool prof) {
  // External records become real event nodes when captured into a graph (a plain record
  // inside a capture is only an intra-graph dependency marker and is never timestamped).
  for (size_t i = 0; i < m->steps.size(); ++i) {
    if (prof) SPINN_CUDA_TRY(cudaEventRecordWithFlags(m->events[i], st, cudaEventRecordExternal));
    int rc = m->steps[i].run(st);
    if (rc) return rc;
  }
  if (prof) SPINN_CUDA_TRY(cudaEventRecordWithFlags(m->events[m->steps.size()], st, cudaEventRecordExternal));
  return 0;
}

static void release_model(SpinnCudaModel* m) {
  if (!m) return;
  if (m->device >= 0) cudaSetDevice(m->device);
  if (m->gexec) cudaGraphExecDestroy(m->gexec);
  if (m->graph) cudaGraphDestroy(m->graph);
  if (m->pgexec) cudaGraphExecDestroy(m->pgexec);
  if (m->pgraph) cudaGraphDestroy(m->pgraph);
  for (auto e : m->events) cudaEventDestroy(e);
  for (auto& b : m->bufs)
    if (b.external && b.ptr && b.alias < 0) cudaFree(b.ptr);
  if (m->arena) cudaFree(m->arena);
  if (m->wdev) cudaFree(m->wdev);
  if (m->splitk_ws) cudaFree(m->splitk_ws);
  if (m->sk_flags) cudaFree(m->sk_flags);
  if (m->copy_stream) cudaStreamSynchronize(m->copy_stream);
  if (m->gexec_alt) cudaGraphExecDestroy(m->gexec_alt);
  if (m->graph_alt) cudaGraphDestroy(m->graph_alt);
  if (m->alt_in) cudaFree(m->alt_in);
  for (int k = 0; k < 2; ++k) {
    if (m->in_ready[k]) cudaEventDestroy(m->in_ready[k]);
    if (m->in_free[k]) cudaEventDestroy(m->in_free[k]);
  }
  if (m->copy_stream) cudaStreamDestroy(m->copy_stream);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

// ------------------------------------------------------------------ C ABI (model level)
extern "C" {

__attribute__((visibility("default"))) SpinnCudaModel* spinn_cuda_load_buffer(const void* data, size_t size) {
  if (!data || size < sizeof(EnnfHeader)) {
    set_error("spinn_cuda_load_buffer: empty image");
    return nullptr;
  }
  auto* m = new SpinnCudaModel();
  m->image.assign((const uint8_t*)data, (const uint8_t*)data + size);
  if (parse_image(m)) {
    delete m;
    return nullptr;
  }
  return m;
}

__attribute__((visibility("default"))) SpinnCudaModel* spinn_cuda_load(const char* path) {
  FILE* f = path ? fopen(path, "rb") : nullptr;
  if (!f) {
    set_error("spinn_cuda_load: cannot open %s", path ? path : "(null)");
    return nullptr;
  }
  fseek(f, 0, SEEK_END);
  const long sz = ftell(f);
  fseek(f, 0, SEEK_SET);
  std::vector<uint8_t> buf(sz > 0 ? sz : 0);
  const size_t rd = sz > 0 ? fread(buf.data(), 1, sz, f) : 0;
  fclose(f);
  if ((long)rd != sz) {
    set_error("spinn_cuda_load: short read on %s", path);
    return nullptr;
  }
  return spinn_cuda_load_buffer(buf.data(), buf.size());
}

__attribute__((visibility("default"))) int spinn_cuda_plan(SpinnCudaModel* m, int device, uint64_t max_arena_bytes,
                                                           int flags) {
  if (!m) {
    set_error("spinn_cuda_plan: null model");
    return SPINN_CUDA_EINVAL;
  }
  if (m->planned) {
    set_error("spinn_cuda_plan: model already planned");
    return SPINN_CUDA_ESTATE;
  }
  SPINN_CUDA_TRY(cudaSetDevice(device));
  m->device = device;
  m->flags = flags;
  SPINN_CUDA_TRY(cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking));
  int rc = compile_model(m, max_arena_bytes);
  if (rc) return rc;
  if (flags & SPINN_CUDA_PLAN_PROFILE) {
    m->events.resize(m->steps.size() + 1);
    for (auto& e : m->events) SPINN_CUDA_TRY(cudaEventCreate(&e));
  }
  // one eager pass validates every launch; then the step list is captured as a graph
  rc = run_steps(m, m->stream, false);
  if (rc) return rc;
  SPINN_CUDA_TRY(cudaStreamSynchronize(m->stream));
  rc = check_run(m, m->stream);
  if (rc) return rc;
  if (!(flags & SPINN_CUDA_PLAN_NO_GRAPH)) {
    for (int pass = 0; pass < ((flags & SPINN_CUDA_PLAN_PROFILE) ? 2 : 1); ++pass) {
      SPINN_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
      rc = run_steps(m, m->stream, pass == 1);
      cudaGraph_t g = nullptr;
      cudaError_t e = cudaStreamEndCapture(m->stream, &g);
      if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
      }
      SPINN_CUDA_TRY(e);
      cudaGraphExec_t ge = nullptr;
      SPINN_CUDA_TRY(cudaGraphInstantiate(&ge, g, 0));
      if (pass == 0) {
        m->graph = g;
        m->gexec = ge;
        // kernels launched per run: the captured graph's kernel nodes (a split-K step, for
        // instance, is two kernels)
        size_t nn = 0;
        SPINN_CUDA_TRY(cudaGraphGetNodes(g, nullptr, &nn));
        std::vector<cudaGraphNode_t> nodes(nn);
        SPINN_CUDA_TRY(cudaGraphGetNodes(g, nodes.data(), &nn));
        int kern = 0;
        for (size_t i = 0; i < nn; ++i) {
          cudaGraphNodeType t;
          SPINN_CUDA_TRY(cudaGraphNodeGetType(nodes[i], &t));
          if (t == cudaGraphNodeTypeKernel) ++kern;
        }
        m->kernels = kern;
      } else {
        m->pgraph = g;
        m->pgexec = ge;
      }
    }
  }
  m->planned = true;
  return 0;
}

// Runs the step list with an event between steps (the event-annotated graph when one was
// captured) and records every step's device time.
extern "C" __attribute__((visibility("default"))) int spinn_cuda_run_profiled(SpinnCudaModel* m, void* stream) {
  if (!m || !m->planned || m->events.empty()) {
    set_error("spinn_cuda_run_profiled: plan with SPINN_CUDA_PLAN_PROFILE first");
    return SPINN_CUDA_ESTATE;
  }
  SPINN_CUDA_TRY(cudaSetDevice(m->device));
  cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
  if (m->pgexec) {
    SPINN_CUDA_TRY(cudaGraphLaunch(m->pgexec, st));
  } else {
    int rc = run_steps(m, st, true);
    if (rc) return rc;
  }
  SPINN_CUDA_TRY(cudaStreamSynchronize(st));
  m->step_ms.assign(m->steps.size(), 0.0f);
  for (size_t i = 0; i < m->steps.size(); ++i)
    SPINN_CUDA_TRY(cudaEventElapsedTime(&m->step_ms[i], m->events[i], m->events[i + 1]));
  return check_run(m, st);
}

__attribute__((visibility("default"))) int spinn_cuda_run_device(SpinnCudaModel* m, void* stream) {
  if (!m || !m->planned) {
    set_error("spinn_cuda_run_device: model not planned");
    return SPINN_CUDA_ESTATE;
  }
  SPINN_CUDA_TRY(cudaSetDevice(m->device));
  cudaStream_t st = stream ? (cudaStream_t)stream : m->stream;
  if (m->gexec) {
    SPINN_CUDA_TRY(cudaGraphLaunch(m->gexec, st));
    return 0;
  }
  return run_steps(m, st, false);
}

__attribute__((visibility("default"))) int spinn_cuda_run(SpinnCudaModel* m, const void* input, void* output) {
  if (!m || !m->planned) {
    set_error("spinn_cuda_run: model not planned");
    return SPINN_CUDA_ESTATE;
  }
  SPINN_CUDA_TRY(cudaSetDevice(m->device));
  if (input && !m->in_buf.empty()) {
    const Buf& b = m->bufs[m->in_buf[0]];
    SPINN_CUDA_TRY(cudaMemcpyAsync(b.ptr, input, b.bytes, cudaMemcpyHostToDevice, m->stream));
  }
  int rc = spinn_cuda_run_device(m, nullptr);
  if (rc) return rc;
  if (output && !m->out_buf.empty()) {
    const Buf& b = m->bufs[m->out_buf[0]];
    SPINN_CUDA_TRY(cudaMemcpyAsync(output, b.ptr, b.bytes, cudaMemcpyDeviceToHost, m->stream));
  }
  SPINN_CUDA_TRY(cudaStreamSynchronize(m->stream));
  return check_run(m, m->stream);
}

// Points input 0 -- its staging buffer and every tensor aliasing it -- at `p`; returns the
// previous address.
static float* set_input0_ptr(SpinnCudaModel* m, float* p) {
  const int sb = m->in_buf[0];
  float* old = m->bufs[sb].ptr;
  for (size_t i = 0; i < m->bufs.size(); ++i) {
    int r = (int)i;
    while (m->bufs[r].alias >= 0) r = m->bufs[r].alias;
    if (r == sb) m->bufs[i].ptr = p;
  }
  return old;
}

// One run of the step list with input 0 read from slot `slot` (0: its own buffer, 1: alt_in).
static int launch_slot(SpinnCudaModel* m, int slot) {
  if (slot == 0 || m->in_buf.empty()) return spinn_cuda_run_device(m, nullptr);
  if (m->gexec_alt) {
    SPINN_CUDA_TRY(cudaGraphLaunch(m->gexec_alt, m->stream));
    return 0;
  }
  float* own = set_input0_ptr(m, reinterpret_cast<float*>(m->alt_in));  // eager mode (no graph)
  const int rc = run_steps(m, m->stream, false);
  set_input0_ptr(m, own);
  return rc;
}

__attribute__((visibility("default"))) int spinn_cuda_submit(SpinnCudaModel* m, const void* input, void* output) {
  if (!m || !m->planned) {
    set_error("spinn_cuda_submit: model not planned");
    return SPINN_CUDA_ESTATE;
  }
  SPINN_CUDA_TRY(cudaSetDevice(m->device));
  int slot = 0;
  if (input && !m->in_buf.empty()) {
    const Buf& b = m->bufs[m->in_buf[0]];
    if (!m->copy_stream) {
      SPINN_CUDA_TRY(cudaStreamSynchronize(m->stream));
      SPINN_CUDA_TRY(cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking));
      for (int k = 0; k < 2; ++k) {
        SPINN_CUDA_TRY(cudaEventCreateWithFlags(&m->in_ready[k], cudaEventDisableTiming));
        SPINN_CUDA_TRY(cudaEventCreateWithFlags(&m->in_free[k], cudaEventDisableTiming));
      }
      SPINN_CUDA_TRY(cudaMalloc(&m->alt_in, align_up(b.bytes, 256)));
      if (m->gexec) {  // the same step list, captured once more with input 0 at alt_in
        float* own = set_input0_ptr(m, reinterpret_cast<float*>(m->alt_in));
        cudaError_t e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
        int rc = e == cudaSuccess ? run_steps(m, m->stream, false) : 0;
        cudaGraph_t g = nullptr;
        if (e == cudaSuccess) e = cudaStreamEndCapture(m->stream, &g);
        set_input0_ptr(m, own);
        if (rc || e != cudaSuccess) {
          if (g) cudaGraphDestroy(g);
          if (rc) return rc;
          SPINN_CUDA_TRY(e);
        }
        m->graph_alt = g;
        SPINN_CUDA_TRY(cudaGraphInstantiate(&m->gexec_alt, g, 0));
      }
    }
    slot = (int)(m->submitted & 1);
    void* dst = slot == 0 ? (void*)b.ptr : m->alt_in;
    // the run that last read this slot (two submissions back) has finished; an event never
    // recorded is no wait
    SPINN_CUDA_TRY(cudaStreamWaitEvent(m->copy_stream, m->in_free[slot], 0));
    SPINN_CUDA_TRY(cudaMemcpyAsync(dst, input, b.bytes, cudaMemcpyHostToDevice, m->copy_stream));
    SPINN_CUDA_TRY(cudaEventRecord(m->in_ready[slot], m->copy_stream));
    SPINN_CUDA_TRY(cudaStreamWaitEvent(m->stream, m->in_ready[slot], 0));
  }
  int rc = launch_slot(m, slot);
  if (rc) return rc;
  if (input && !m->in_buf.empty()) SPINN_CUDA_TRY(cudaEventRecord(m->in_free[slot], m->stream));
  if (output && !m->out_buf.empty()) {
    const Buf& b = m->bufs[m->out_buf[0]];
    SPINN_CUDA_TRY(cudaMemcpyAsync(output, b.ptr, b.bytes, cudaMemcpyDeviceToHost, m->stream));
  }
  ++m->submitted;
  return 0;
}

__attribute__((visibility("default"))) int spinn_cuda_wait(SpinnCudaModel* m) {
  if (!m || !m->planned) {
    set_error("spinn_cuda_wait: model not planned");
    return SPINN_CUDA_ESTATE;
  }
  SPINN_CUDA_TRY(cudaSetDevice(m->device));
  SPINN_CUDA_TRY(cudaStreamSynchronize(m->stream));
  return check_run(m, m->stream);
}

__attribute__((visibility("default"))) void* spinn_cuda_io_ptr(SpinnCudaModel* m, int is_output, int index,
                                                               size_t* bytes) {
  if (!m || !m->planned) return nullptr;
  const auto& v = is_output ? m->out_buf : m->in_buf;
  if (index < 0 || index >= (int)v.size()) return nullptr;
  const Buf& b = m->bufs[v[index]];
  if (bytes) *bytes = b.bytes;
  return b.ptr;
}

__attribute__((visibility("default"))) int spinn_cuda_io_count(SpinnCudaModel* m, int is_output) {
  if (!m) return SPINN_CUDA_EINVAL;
  return (int)(is_output ? m->outputs.size() : m->inputs.size());
}

__attribute__((visibility("default"))) int spinn_cuda_io_dims(SpinnCudaModel* m, int is_output, int index,
                                                              uint32_t* dims) {
  if (!m) return SPINN_CUDA_EINVAL;
  const auto& v = is_output ? m->outputs : m->inputs;
  if (index < 0 || index >= (int)v.size()) return SPINN_CUDA_EINVAL;
  const TensorRec& t = m->tensors[v[index]];
  if (dims) std::memcpy(dims, t.dims, sizeof(t.dims));
  return t.ndim;
}

__attribute__((visibility("default"))) int spinn_cuda_io_dtype(SpinnCudaModel* m, int is_output, int index) {
  if (!m) return SPINN_CUDA_EINVAL;
  const auto& v = is_output ? m->outputs : m->inputs;
  if (index < 0 || index >= (int)v.size()) return SPINN_CUDA_EINVAL;
  return m->tensors[v[index]].dtype == kDtypeInt64 ? kDtypeInt64 : 1;
}

__attribute__((visibility("default"))) int spinn_cuda_copy_output(SpinnCudaModel* m, int index, void* host,
                                                                  size_t bytes) {
  if (!m || !m->planned || !host) {
    set_error("spinn_cuda_copy_output: model not planned or no host buffer");
    return SPINN_CUDA_ESTATE;
  }
  if (index < 0 || index >= (int)m->out_buf.size()) {
    set_error("spinn_cuda_copy_output: output %d of %d", index, (int)m->out_buf.size());
    return SPINN_CUDA_EINVAL;
  }
  const Buf& b = m->bufs[m->out_buf[index]];
  if (bytes != b.bytes) {
    set_error("spinn_cuda_copy_output: output %d has %llu bytes, not %zu", index, (unsigned long long)b.bytes,
              bytes);
    return SPINN_CUDA_EINVAL;
  }
  SPINN_CUDA_TRY(cudaSetDevice(m->device));
  SPINN_CUDA_TRY(cudaMemcpyAsync(host, b.ptr, bytes, cudaMemcpyDeviceToHost, m->stream));
  SPINN_CUDA_TRY(cudaStreamSynchronize(m->stream));
  return 0;
}

__attribute__((visibility("default"))) int spinn_cuda_copy_tensor(SpinnCudaModel* m, int tensor_id, int first,
                                                                  int count, void* host, size_t bytes) {
  if (!m || !m->planned || !host) {
    set_error("spinn_cuda_copy_tensor: model not planned or no host buffer");
    return SPINN_CUDA_ESTATE;
  }
  if (tensor_id < 0 || tensor_id >= (int)m->tensors.size() || tensor_id >= (int)m->bufs.size()) {
    set_error("spinn_cuda_copy_tensor: no tensor %d", tensor_id);
    return SPINN_CUDA_EINVAL;
  }
  const TensorRec& t = m->tensors[tensor_id];
  const bool is_output = std::find(m->outputs.begin(), m->outputs.end(), (uint16_t)tensor_id) != m->outputs.end();
  if (!(m->flags & SPINN_CUDA_PLAN_KEEP) && !is_output) {
    set_error("spinn_cuda_copy_tensor: tensor %d is not a graph output; plan with SPINN_CUDA_PLAN_KEEP", tensor_id);
    return SPINN_CUDA_ESTATE;
  }
  // views without storage of their own: a Reshape to [N, C, H*W] gathered from its NHWC input
  // has that input's NCHW bytes; a Transpose folded into a MatMul is its input transposed
  auto lz = m->lazy_nchw.find(tensor_id);
  if (lz != m->lazy_nchw.end()) return spinn_cuda_copy_tensor(m, lz->second, first, count, host, bytes);
  auto bt = m->b_trans.find(tensor_id);
  if (bt != m->b_trans.end()) {
    const TensorRec& x = m->tensors[bt->second];
    if (x.ndim < 2 || bytes % 4) {
      set_error("spinn_cuda_copy_tensor: tensor %d is a folded transpose of a tensor below 2-D", tensor_id);
      return SPINN_CUDA_EINVAL;
    }
    std::vector<float> tmp(bytes / 4);
    const int rc = spinn_cuda_copy_tensor(m, bt->second, first, count, tmp.data(), bytes);
    if (rc) return rc;
    const uint64_t rows = x.dims[x.ndim - 2], cols = x.dims[x.ndim - 1], plane = rows * cols;
    float* dst = static_cast<float*>(host);
    for (uint64_t p0 = 0; plane && p0 + plane <= tmp.size(); p0 += plane)
      for (uint64_t r = 0; r < rows; ++r)
        for (uint64_t c = 0; c < cols; ++c) dst[p0 + c * rows + r] = tmp[p0 + r * cols + c];
    return 0;
  }
  int r = tensor_id;
  while (m->bufs[r].alias >= 0) r = m->bufs[r].alias;
  const Buf& b = m->bufs[tensor_id];
  const float* base = m->bufs[r].ptr;
  auto vc = m->virt_cat.find(tensor_id);
  if (vc != m->virt_cat.end() && t.ndim == 4 && first >= 0 && count >= 1 &&
      (uint64_t)first + count <= t.dims[0] && bytes == (uint64_t)count * (t.elems / t.dims[0]) * 4) {
    // a Concat read in parts by its convolution: gather the parts (NCHW, channel after channel)
    SPINN_CUDA_TRY(cudaSetDevice(m->device));
    SPINN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    const uint64_t hw = (uint64_t)t.dims[2] * t.dims[3];
    float* dst = static_cast<float*>(host);
    int c0 = 0;
    for (int pbi : vc->second) {
      const Buf& pb = m->bufs[pbi];
      const uint64_t img = hw * pb.cpad;
      std::vector<float> tmp((size_t)(count * img));
      SPINN_CUDA_TRY(cudaMemcpy(tmp.data(), pb.ptr + (uint64_t)first * img, tmp.size() * 4, cudaMemcpyDeviceToHost));
      for (int n = 0; n < count; ++n)
        for (int c = 0; c < pb.c; ++c)
          for (uint64_t q = 0; q < hw; ++q)
            dst[((uint64_t)n * t.dims[1] + c0 + c) * hw + q] = tmp[n * img + q * pb.cpad + c];
      c0 += pb.c;
    }
    return 0;
  }
  if (t.is_weight || !base || b.lay == LAY_NONE || t.ndim < 1 || t.dims[0] == 0) {
    set_error("spinn_cuda_copy_tensor: tensor %d has no device buffer (weight, fused away or unused)", tensor_id);
    return SPINN_CUDA_EINVAL;
  }
  const uint64_t d0 = t.dims[0];
  if (first < 0 || count < 1 || (uint64_t)first + (uint64_t)count > d0) {
    set_error("spinn_cuda_copy_tensor: items [%d, %d) outside dim 0 = %llu", first, first + count,
              (unsigned long long)d0);
    return SPINN_CUDA_EINVAL;
  }
  const uint64_t esz = elem_bytes(t);
  const uint64_t item_elems = t.elems / d0;
  if (bytes != (uint64_t)count * item_elems * esz) {
    set_error("spinn_cuda_copy_tensor: %d items of tensor %d are %llu bytes, not %zu", count, tensor_id,
              (unsigned long long)((uint64_t)count * item_elems * esz), bytes);
    return SPINN_CUDA_EINVAL;
  }
  SPINN_CUDA_TRY(cudaSetDevice(m->device));
  SPINN_CUDA_TRY(cudaStreamSynchronize(m->stream));
  if (b.lay == LAY_NHWC) {
    // NHWC with padded channels on the device -> NCHW on the host
    const uint64_t hw = (uint64_t)b.h * b.w, img = hw * b.cpad;
    std::vector<float> tmp((size_t)(count * img));
    SPINN_CUDA_TRY(cudaMemcpy(tmp.data(), base + (uint64_t)first * img, tmp.size() * 4, cudaMemcpyDeviceToHost));
    float* dst = static_cast<float*>(host);
    for (int n = 0; n < count; ++n)
      for (int c = 0; c < b.c; ++c)
        for (uint64_t p = 0; p < hw; ++p) dst[((uint64_t)n * b.c + c) * hw + p] = tmp[n * img + p * b.cpad + c];
  } else {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(base) + (uint64_t)first * item_elems * esz;
    SPINN_CUDA_TRY(cudaMemcpy(host, src, bytes, cudaMemcpyDeviceToHost));
  }
  return 0;
}

__attribute__((visibility("default"))) int spinn_cuda_plan_info(SpinnCudaModel* m, uint64_t* arena_bytes,
                                                                uint64_t* weight_bytes, int* num_steps,
                                                                int* num_kernels) {
  if (!m || !m->planned) return SPINN_CUDA_ESTATE;
  if (arena_bytes) *arena_bytes = m->arena_bytes;
  if (weight_bytes) *weight_bytes = m->wbytes;
  if (num_steps) *num_steps = (int)m->steps.size();
  if (num_kernels) *num_kernels = m->kernels;
  return 0;
}

__attribute__((visibility("default"))) int spinn_cuda_profile(SpinnCudaModel* m, int* op_types, float* ms,
                                                              double* flops, int cap) {
  if (!m || !m->planned) return SPINN_CUDA_ESTATE;
  const int n = std::min<int>(cap, (int)m->step_ms.size());
  for (int i = 0; i < n; ++i) {
    if (op_types) op_types[i] = m->steps[i].op;
    if (ms) ms[i] = m->step_ms[i];
    if (flops) flops[i] = m->steps[i].flops;
  }
  return n;
}

__attribute__((visibility("default"))) int spinn_cuda_step_kind(SpinnCudaModel* m, int i) {
  if (!m || i < 0 || i >= (int)m->steps.size()) return -1;
  return m->steps[i].kind;
}

__attribute__((visibility("default"))) void spinn_cuda_free(SpinnCudaModel* m) { release_model(m); }

}  // extern "C"
}  // namespace spinn
