// loader.cpp — the converted AR checkpoint into HBM (ARModel::ARModel,
// native/src/ar.cpp:133-238, with verify=false as Pipeline::load_ar calls it,
// native/src/pipeline.cpp:131-176).
//
// Checks, in the reference's order and with its error types:
//   1. conversion.json is a schema-1 manifest with a record for the precision: bf16 names
//      ar-bf16.safetensors and dtype bfloat16; 8bit / 4bit name ar-8bit / ar-4bit
//      .safetensors with bits 8 / 4, group_size 64, mode affine, linear_only (ar.cpp:137-160)
//   2. config.json matches the pinned generator config             (ar.cpp:161-192)
//   3. the AR file holds exactly the AR tensor set with the pinned shapes: BF16, or for
//      8bit / 4bit every linear as a U32 [out, in * bits / 32] weight with BF16 [out, in / 64] scales
//      and biases                                                  (ar.cpp:193-236)
// Quantized weights are dequantized on the GPU into the BF16 layout below (prefill and the
// batched and per-operation decode paths read it) and also written as the stage images
// the persistent decode kernel streams (Model::qarena).
// Device layout (one allocation): per layer the q/k/v rows stacked into one [q+2kv][H]
// matrix, gate/up rows interleaved (row 2j gate j, row 2j+1 up j) so a SwiGLU output
// comes from one row pair, and everything else as stored (row-major [out][in]).
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <map>
#include <set>
#include <sstream>

#include "engine.h"
#include "exact_math.cuh"
#include "nlohmann/json.hpp"

namespace yar {

using Json = nlohmann::json;

void throw_cuda(cudaError_t e, const char *what, const char *file, int line) {
  std::ostringstream os;
  os << "CUDA error " << cudaGetErrorName(e) << " (" << cudaGetErrorString(e) << ") at " << file << ":"
     << line << ": " << what;
  throw Error("RuntimeError", os.str());
}

static Json read_json(const std::string &path) {
  std::ifstream in(path);
  if (!in) throw Error("FileNotFoundError", "Missing file: " + path);
  std::stringstream ss;
  ss << in.rdbuf();
  try {
    return Json::parse(ss.str());
  } catch (const std::exception &e) {
    throw Error("ValueError", "Invalid JSON in " + path + ": " + e.what());
  }
}

PhaseRows phase_rows(const Dims &d, int phase) {
  PhaseRows r;
  if (phase == kPhaseFull) {
    r.row0 = 0;
    r.n_main = d.vocab;
    return r;
  }
  if (d.vocab != 184704) throw Error("ValueError", "Protocol phases need the 184704-row vocabulary");
  if (phase == kPhaseAbc) {
    r.row0 = 0;
    r.n_main = kEOD;
    r.extra = kAbcEnd;
  } else if (phase == kPhaseSemantic) {
    r.row0 = kMusicEnd;
    r.n_main = kCodecOffset + kCodecSize - kMusicEnd;
  } else {
    throw Error("ValueError", "phase must be 'abc' or 'semantic'");
  }
  return r;
}

static Dims config_dims(const Json &config, bool any_dims) {
  if (!config.is_object()) throw Error("ValueError", "config.json must contain a JSON object");
  const std::vector<std::pair<std::string, Json>> pinned = {
      {"hidden_size", 2048},      {"intermediate_size", 6144},        {"num_hidden_layers", 28},
      {"num_attention_heads", 16}, {"num_key_value_heads", 8},         {"head_dim", 128},
      {"vocab_size", 184704},     {"max_position_embeddings", kContext}, {"rope_theta", 1000000.0}};
  for (const auto &[key, expected] : pinned) {
    Json actual = config.contains(key) ? config[key]
                                        : (key == "max_position_embeddings" ? Json(kContext) : Json());
    if (!any_dims && actual != expected) throw Error("ValueError", "Incompatible YuE2 config: " + key);
    if (key != "rope_theta" && !(actual.is_number_integer() && actual.get<long long>() > 0))
      throw Error("ValueError", "Generator config field " + key + " must be a positive integer");
    if (key == "rope_theta" && !(actual.is_number() && actual.get<double>() > 0))
      throw Error("ValueError", "rope_theta must be a positive number");
  }
  if (config.value("tie_word_embeddings", Json(false)) != Json(false))
    throw Error("ValueError", "YuE2 requires untied input and output embeddings");
  if (config.contains("rope_scaling") && !config["rope_scaling"].is_null() &&
      config["rope_scaling"] != Json::object())
    throw Error("ValueError", "YuE2 uses fixed base RoPE without scaling");
  if (config.value("hidden_act", std::string("silu")) != "silu")
    throw Error("ValueError", "Incompatible YuE2 config: hidden_act must be silu");
  if (!config.contains("rms_norm_eps") || !config["rms_norm_eps"].is_number() ||
      !std::isfinite(config["rms_norm_eps"].get<double>()) || config["rms_norm_eps"].get<double>() <= 0)
    throw Error("ValueError", "rms_norm_eps must be finite and positive");
  Dims d;
  d.hidden = config["hidden_size"];
  d.ffn = config["intermediate_size"];
  d.layers = config["num_hidden_layers"];
  d.heads = config["num_attention_heads"];
  d.kv_heads = config["num_key_value_heads"];
  d.head_dim = config["head_dim"];
  d.vocab = config["vocab_size"];
  d.context = config.value("max_position_embeddings", kContext);
  d.theta = config["rope_theta"].get<double>();
  d.eps = float(config["rms_norm_eps"].get<double>());
  if (d.heads % d.kv_heads != 0) throw Error("ValueError", "num_attention_heads must be a multiple of num_key_value_heads");
  if (d.head_dim != 64 && d.head_dim != 128) throw Error("ValueError", "head_dim must be 64 or 128");
  if (d.hidden % 8 || d.ffn % 8) throw Error("ValueError", "hidden_size and intermediate_size must be multiples of 8");
  if (d.context > kContext) throw Error("ValueError", "max_position_embeddings above 24576");
  return d;
}

struct TensorRec {
  std::vector<int64_t> shape;
  uint64_t begin, end;
  std::string dtype;  // "BF16" or "U32"
};

static std::map<std::string, TensorRec> read_safetensors_header(const std::string &path, uint64_t &data_start) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw Error("FileNotFoundError", "Converted artifact does not contain its AR weights file: " + path);
  in.seekg(0, std::ios::end);
  const uint64_t size = uint64_t(in.tellg());
  in.seekg(0);
  uint64_t len = 0;
  if (size < 10) throw Error("ValueError", "Invalid safetensors file: " + path);
  in.read(reinterpret_cast<char *>(&len), 8);
  if (!in || len < 2 || len > 64ull * 1024 * 1024 || len > size - 8)
    throw Error("ValueError", "Invalid safetensors header size");
  std::string raw(len, '\0');
  in.read(raw.data(), std::streamsize(len));
  if (!in) throw Error("ValueError", "Truncated safetensors header");
  Json h;
  try {
    h = Json::parse(raw);
  } catch (const std::exception &e) {
    throw Error("ValueError", std::string("Invalid safetensors header: ") + e.what());
  }
  if (!h.is_object()) throw Error("ValueError", "Invalid safetensors header");
  data_start = 8 + len;
  std::map<std::string, TensorRec> out;
  for (auto it = h.begin(); it != h.end(); ++it) {
    if (it.key() == "__metadata__") continue;
    const Json &r = it.value();
    if (!r.is_object() || !r.contains("dtype") || !r.contains("shape") || !r.contains("data_offsets"))
      throw Error("ValueError", "Invalid safetensors entry: " + it.key());
    if (r["dtype"] != "BF16" && r["dtype"] != "U32")
      throw Error("ValueError", "Incompatible AR tensor shape/dtype: " + it.key());
    TensorRec t;
    t.dtype = r["dtype"].get<std::string>();
    for (const auto &v : r["shape"]) t.shape.push_back(v.get<int64_t>());
    t.begin = r["data_offsets"][0].get<uint64_t>();
    t.end = r["data_offsets"][1].get<uint64_t>();
    uint64_t n = t.dtype == "U32" ? 4 : 2;
    for (auto v : t.shape) n *= uint64_t(v);
    if (t.end < t.begin || t.end - t.begin != n || data_start + t.end > size)
      throw Error("ValueError", "Truncated or inconsistent safetensors tensor: " + it.key());
    out.emplace(it.key(), std::move(t));
  }
  return out;
}

TpPlan tp_plan(const Dims &d, int rank, int world) {
  if (world < 1 || rank < 0 || rank >= world) throw Error("ValueError", "tensor-parallel rank outside [0, world)");
  if (d.kv_heads % world || d.ffn % world || (d.ffn / world) % 8 || d.hidden % (8 * world))
    throw Error("ValueError",
                "tensor-parallel world must divide num_key_value_heads, intermediate_size / 8 and hidden_size / 8");
  const int group = d.heads / d.kv_heads;  // query heads per KV head stay together
  TpPlan p;
  p.kv_rows = d.kv_heads / world * d.head_dim;
  p.kv_row0 = rank * p.kv_rows;
  p.q_rows = p.kv_rows * group;
  p.q_row0 = rank * p.q_rows;
  p.ffn_rows = d.ffn / world;
  p.ffn_row0 = rank * p.ffn_rows;
  p.h_rows = d.hidden / world;
  p.h_row0 = rank * p.h_rows;
  return p;
}

Model *load_model(const std::string &dir, int device, uint32_t flags, int tp_rank, int tp_world,
                  const uint8_t *nccl_id) {
  const bool any_dims = flags & 1u;
  if ((flags & 2u) && (flags & 4u)) throw Error("ValueError", "choose one of 8-bit and 4-bit weights");
  // YAR_LOAD_8BIT / YAR_LOAD_4BIT: the `8bit` / `4bit` precision.
  const int bits = (flags & 2u) ? 8 : (flags & 4u) ? 4 : 0;
  const std::string precision = bits ? std::to_string(bits) + "bit" : "bf16";
  if (tp_world > 1 && !nccl_id) throw Error("ValueError", "tensor parallelism needs an NCCL unique id");
  if (tp_world > 1 && bits) throw Error("ValueError", "quantized AR weights are not built for tensor parallelism");
  // 1. Manifest.
  Json manifest = read_json(dir + "/conversion.json");
  if (!manifest.is_object() || manifest.value("schema", 0) != 1)
    throw Error("ValueError", "conversion.json must be a schema-1 manifest");
  if (!manifest.contains("precisions") || !manifest["precisions"].is_object() ||
      !manifest["precisions"].contains(precision) || !manifest["precisions"][precision].is_object())
    throw Error("FileNotFoundError", "Converted artifact does not contain " + precision + " AR weights");
  const Json &entry = manifest["precisions"][precision];
  const std::string filename = "ar-" + precision + ".safetensors";
  if (entry.value("ar", std::string()) != filename)
    throw Error("ValueError", "Manifest AR filename does not match precision");
  if (!bits) {
    if (entry.value("dtype", std::string()) != "bfloat16")
      throw Error("ValueError", "BF16 manifest entry must declare dtype='bfloat16'");
  } else if (entry.value("bits", 0) != bits || entry.value("group_size", 0) != 64 ||
             entry.value("mode", std::string()) != "affine" || entry.value("linear_only", false) != true) {
    throw Error("ValueError", "Invalid affine quantization settings in AR manifest");
  }
  // 2. Config.
  const Dims d = config_dims(read_json(dir + "/config.json"), any_dims);
  if (bits && (d.hidden % 64 || d.ffn % 64 || d.qdim() % 64))
    throw Error("ValueError", "quantized AR weights need every linear's input width to be a multiple of 64");
  // 3. Tensors.
  const std::string path = dir + "/" + filename;
  uint64_t data_start = 0;
  auto recs = read_safetensors_header(path, data_start);
  std::set<std::string> expected;
  auto require = [&](const std::string &name, std::vector<int64_t> shape, const char *dtype = "BF16") {
    expected.insert(name);
    auto it = recs.find(name);
    if (it == recs.end()) throw Error("ValueError", "Missing AR tensor: " + name);
    if (it->second.shape != shape || it->second.dtype != dtype)
      throw Error("ValueError", "Incompatible AR tensor shape/dtype: " + name);
  };
  // A linear layer's tensors (ar.cpp:208-214): the BF16 weight, or the packed quantized form.
  auto require_linear = [&](const std::string &n, int64_t out, int64_t in) {
    if (!bits) {
      require(n + ".weight", {out, in});
      return;
    }
    require(n + ".weight", {out, in * bits / 32}, "U32");
    require(n + ".scales", {out, in / 64});
    require(n + ".biases", {out, in / 64});
  };
  const int H = d.hidden, Q = d.qdim(), KV = d.kvdim(), F = d.ffn, V = d.vocab, D = d.head_dim;
  require("model.embed_tokens.weight", {V, H});
  require("model.norm.weight", {H});
  require_linear("lm_head", V, H);
  for (int i = 0; i < d.layers; ++i) {
    const std::string n = "model.layers." + std::to_string(i), a = n + ".self_attn";
    require(n + ".input_layernorm.weight", {H});
    require(n + ".post_attention_layernorm.weight", {H});
    require(a + ".q_norm.weight", {D});
    require(a + ".k_norm.weight", {D});
    require_linear(a + ".q_proj", Q, H);
    require_linear(a + ".k_proj", KV, H);
    require_linear(a + ".v_proj", KV, H);
    require_linear(a + ".o_proj", H, Q);
    require_linear(n + ".mlp.gate_proj", F, H);
    require_linear(n + ".mlp.up_proj", F, H);
    require_linear(n + ".mlp.down_proj", H, F);
  }
  for (const auto &[name, rec] : recs)
    if (!expected.count(name)) throw Error("ValueError", "Unexpected AR tensor: " + name);
  // Tensor-parallel share of this rank (the tensors keep their full shapes on disk).
  const TpPlan plan = tp_plan(d, tp_rank, tp_world);
  Dims dl = d;
  dl.heads = plan.q_rows / d.head_dim;
  dl.kv_heads = plan.kv_rows / d.head_dim;
  dl.ffn = plan.ffn_rows;
  const int Ql = dl.qdim(), KVl = dl.kvdim(), Fl = dl.ffn, Hs = plan.h_rows;

  // Arena layout (256-byte aligned pieces).
  auto *m = new Model();
  try {
    m->d = dl;
    m->full = d;
    m->tp_rank = tp_rank;
    m->tp_world = tp_world;
    m->tp = plan;
    m->device = device;
    YAR_CUDA(cudaSetDevice(device));
    YAR_CUDA(cudaDeviceGetAttribute(&m->sm_count, cudaDevAttrMultiProcessorCount, device));
    configure_gemv_kernels();
    configure_gemm_kernels();
    configure_attn_kernels();
    configure_attn_tc_kernels();
    configure_gemv_tma_kernels();
    configure_persistent_kernels();
    configure_sampler_kernels();
    configure_gemm_tc_kernels();
    size_t off = 0;
    auto take = [&](size_t bytes) {
      const size_t o = off;
      off = (off + bytes + 255) & ~size_t(255);
      return o;
    };
    const size_t e2 = sizeof(uint16_t);
    const size_t o_embed = take(size_t(V) * H * e2), o_head = take(size_t(V) * H * e2), o_norm = take(size_t(H) * e2);
    struct LO { size_t qkv, o, gu, down, ln1, ln2, qn, kn; };
    std::vector<LO> lo(d.layers);
    for (int i = 0; i < d.layers; ++i) {
      lo[i].qkv = take(size_t(Ql + 2 * KVl) * H * e2);
      lo[i].o = take(size_t(Hs) * Q * e2);
      lo[i].gu = take(size_t(2 * Fl) * H * e2);
      lo[i].down = take(size_t(Hs) * F * e2);
      lo[i].ln1 = take(H * e2);
      lo[i].ln2 = take(H * e2);
      lo[i].qn = take(D * e2);
      lo[i].kn = take(D * e2);
    }
    const size_t o_cos = take(size_t(d.context) * (D / 2) * 4), o_sin = take(size_t(d.context) * (D / 2) * 4);
    m->arena_bytes = off;
    YAR_CUDA(cudaMalloc(&m->arena, off));
    char *base = static_cast<char *>(m->arena);
    auto at = [&](size_t o) { return reinterpret_cast<bf16 *>(base + o); };

    // Quantized: the stage images (m->qarena; only when every K is a multiple of 2048, the
    // persistent kernel's stage width) and the raw buffers of one fused matrix (freed when
    // the load ends).
    struct DevBuf {
      void *p = nullptr;
      ~DevBuf() {
        if (p) cudaFree(p);
      }
    } raw_qb, raw_sb, raw_bb;
    struct QLO { size_t qkv, o, gu, down; };
    std::vector<QLO> qlo(d.layers);
    size_t qh_off[3] = {SIZE_MAX, SIZE_MAX, SIZE_MAX};
    unsigned char *qbase = nullptr;
    char *raw_q = nullptr;
    uint16_t *raw_s = nullptr, *raw_b = nullptr;
    if (bits) {
      m->bits = bits;
      if (H % 2048 == 0 && Q % 2048 == 0 && F % 2048 == 0) {
        size_t qoff = 0;
        auto qtake = [&](size_t bytes) {
          const size_t o = qoff;
          qoff = (qoff + bytes + 1023) & ~size_t(1023);
          return o;
        };
        for (int i = 0; i < d.layers; ++i) {
          qlo[i].qkv = qtake(q_image_bytes(Q + 2 * KV, H, bits));
          qlo[i].o = qtake(q_image_bytes(H, Q, bits));
          qlo[i].gu = qtake(q_image_bytes(2 * F, H, bits));
          qlo[i].down = qtake(q_image_bytes(H, F, bits));
        }
        const bool pinned_vocab = V == 184704;  // the protocol phases; otherwise the whole vocabulary
        for (int ph : {kPhaseAbc, kPhaseSemantic, kPhaseFull}) {
          if ((ph == kPhaseFull) == pinned_vocab) continue;
          qh_off[ph] = qtake(q_image_bytes(phase_rows(d, ph).n_main, H, bits));
        }
        m->qarena_bytes = qoff;
        YAR_CUDA(cudaMalloc(&m->qarena, qoff));
        qbase = static_cast<unsigned char *>(m->qarena);
        m->qlayers.resize(d.layers);
      }
      const size_t max_nk = std::max({size_t(Q + 2 * KV) * H, size_t(H) * Q, size_t(2 * F) * H, size_t(H) * F,
                                      size_t(V) * H});
      YAR_CUDA(cudaMalloc(&raw_qb.p, max_nk));
      YAR_CUDA(cudaMalloc(&raw_sb.p, max_nk / 64 * 2));
      YAR_CUDA(cudaMalloc(&raw_bb.p, max_nk / 64 * 2));
      raw_q = static_cast<char *>(raw_qb.p);
      raw_s = static_cast<uint16_t *>(raw_sb.p);
      raw_b = static_cast<uint16_t *>(raw_bb.p);
    }

    // Stream the file through a pinned staging buffer.
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw Error("FileNotFoundError", "Cannot open " + path);
    const size_t stage_bytes = 64ull << 20;
    void *stage = nullptr;
    YAR_CUDA(cudaMallocHost(&stage, 2 * stage_bytes));
    cudaStream_t st;
    YAR_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
    cudaEvent_t done[2];
    YAR_CUDA(cudaEventCreate(&done[0]));
    YAR_CUDA(cudaEventCreate(&done[1]));
    int buf = 0;
    bool pending[2] = {false, false};
    auto pread_all = [&](char *dst, uint64_t file_off, size_t n) {
      size_t got = 0;
      while (got < n) {
        const ssize_t r = ::pread(fd, dst + got, n - got, off_t(file_off + got));
        if (r <= 0) throw Error("ValueError", "Truncated safetensors data in " + path);
        got += size_t(r);
      }
    };
    // Copy the block rows [row0, row0+nrows) x columns [col0, col0+ncols) of a 2-D tensor
    // (a 1-D tensor is one row) to dst, packed [nrows][ncols]; the whole tensor by default.
    auto upload_block = [&](const std::string &name, char *dst, int64_t row0, int64_t nrows, int64_t col0,
                            int64_t ncols) {
      const TensorRec &r = recs.at(name);
      const int64_t cols = r.shape.size() == 2 ? r.shape[1] : r.shape[0];
      const size_t src_row = size_t(cols) * e2, dst_row = size_t(ncols) * e2;
      const bool whole_rows = col0 == 0 && ncols == cols;
      const int64_t rows_per = int64_t(stage_bytes / src_row);
      std::vector<char> tmp(whole_rows ? 0 : size_t(rows_per) * src_row);
      for (int64_t r0 = 0; r0 < nrows; r0 += rows_per) {
        const int64_t nr = std::min(rows_per, nrows - r0);
        if (pending[buf]) YAR_CUDA(cudaEventSynchronize(done[buf]));
        char *sb = static_cast<char *>(stage) + buf * stage_bytes;
        const uint64_t src = data_start + r.begin + uint64_t(row0 + r0) * src_row;
        if (whole_rows) {
          pread_all(sb, src, size_t(nr) * src_row);
        } else {
          pread_all(tmp.data(), src, size_t(nr) * src_row);
          for (int64_t j = 0; j < nr; ++j)
            std::memcpy(sb + size_t(j) * dst_row, tmp.data() + size_t(j) * src_row + size_t(col0) * e2, dst_row);
        }
        YAR_CUDA(cudaMemcpyAsync(dst + size_t(r0) * dst_row, sb, size_t(nr) * dst_row, cudaMemcpyHostToDevice, st));
        YAR_CUDA(cudaEventRecord(done[buf], st));
        pending[buf] = true;
        buf ^= 1;
      }
    };
    auto upload = [&](const std::string &name, char *dst) {
      const TensorRec &r = recs.at(name);
      const int64_t rows = r.shape.size() == 2 ? r.shape[0] : 1, cols = r.shape.size() == 2 ? r.shape[1] : r.shape[0];
      upload_block(name, dst, 0, rows, 0, cols);
    };
    // Interleave gate/up rows into dst: rows 2j (gate j) and 2j+1 (up j).
    // Rows [f0, f0 + nf) of gate_proj and up_proj (this rank's FFN block).
    auto upload_gate_up = [&](const std::string &gate, const std::string &up, char *dst, int f0, int nf) {
      const size_t row_bytes = size_t(H) * e2;
      const size_t rows_per = stage_bytes / (2 * row_bytes);
      for (int r0 = 0; r0 < nf; r0 += int(rows_per)) {
        const int nr = int(std::min<size_t>(rows_per, size_t(nf - r0)));
        if (pending[buf]) YAR_CUDA(cudaEventSynchronize(done[buf]));
        char *sb = static_cast<char *>(stage) + buf * stage_bytes;
        std::vector<char> g(nr * row_bytes), u(nr * row_bytes);
        pread_all(g.data(), data_start + recs.at(gate).begin + size_t(f0 + r0) * row_bytes, g.size());
        pread_all(u.data(), data_start + recs.at(up).begin + size_t(f0 + r0) * row_bytes, u.size());
        for (int j = 0; j < nr; ++j) {
          std::memcpy(sb + (2 * size_t(j)) * row_bytes, g.data() + size_t(j) * row_bytes, row_bytes);
          std::memcpy(sb + (2 * size_t(j) + 1) * row_bytes, u.data() + size_t(j) * row_bytes, row_bytes);
        }
        YAR_CUDA(cudaMemcpyAsync(dst + 2 * size_t(r0) * row_bytes, sb, 2 * size_t(nr) * row_bytes,
                                 cudaMemcpyHostToDevice, st));
        YAR_CUDA(cudaEventRecord(done[buf], st));
        pending[buf] = true;
        buf ^= 1;
      }
    };
    // Quantized: whole rows of a tensor into device memory with a destination row pitch (the
    // rows of one fused matrix: q/k/v stacked, gate/up interleaved).
    auto upload_rows = [&](const std::string &name, int64_t row0, int64_t nrows, char *dst, size_t dst_pitch) {
      const TensorRec &r = recs.at(name);
      const size_t row_bytes = size_t(r.shape[1]) * (r.dtype == "U32" ? 4 : 2);
      const int64_t rows_per = int64_t(stage_bytes / row_bytes);
      for (int64_t r0 = 0; r0 < nrows; r0 += rows_per) {
        const int64_t nr = std::min(rows_per, nrows - r0);
        if (pending[buf]) YAR_CUDA(cudaEventSynchronize(done[buf]));
        char *sb = static_cast<char *>(stage) + buf * stage_bytes;
        pread_all(sb, data_start + r.begin + uint64_t(row0 + r0) * row_bytes, size_t(nr) * row_bytes);
        YAR_CUDA(cudaMemcpy2DAsync(dst + size_t(r0) * dst_pitch, dst_pitch, sb, row_bytes, row_bytes, size_t(nr),
                                   cudaMemcpyHostToDevice, st));
        YAR_CUDA(cudaEventRecord(done[buf], st));
        pending[buf] = true;
        buf ^= 1;
      }
    };
    // A linear's q bytes, scales and biases (rows [row0, row0 + nrows)) into the raw
    // buffers at fused row `dst_row`, every `stride`-th row.
    auto upload_q8 = [&](const std::string &lin, int64_t row0, int64_t nrows, int K, int64_t dst_row, int stride) {
      const size_t qrow = size_t(K) * bits / 8, srow = size_t(K / 64) * 2;
      upload_rows(lin + ".weight", row0, nrows, raw_q + size_t(dst_row) * qrow, stride * qrow);
      upload_rows(lin + ".scales", row0, nrows, reinterpret_cast<char *>(raw_s) + size_t(dst_row) * srow, stride * srow);
      upload_rows(lin + ".biases", row0, nrows, reinterpret_cast<char *>(raw_b) + size_t(dst_row) * srow, stride * srow);
    };
    // The raw fused matrix (N x K) into BF16 weights at `dst` and a stage image at `img`.
    auto finish_q8 = [&](int N, int K, char *dst, unsigned char *img) {
      launch_q_dequant(reinterpret_cast<const uint8_t *>(raw_q), raw_s, raw_b, N, K, bits, reinterpret_cast<bf16 *>(dst),
                       st);
      if (img) launch_q_image(reinterpret_cast<const uint8_t *>(raw_q), raw_s, raw_b, N, K, bits, img, st);
      // The raw buffers are refilled next: wait for these kernels (and the copies before).
      YAR_CUDA(cudaStreamSynchronize(st));
      pending[0] = pending[1] = false;
    };
    upload("model.embed_tokens.weight", base + o_embed);
    if (!bits) {
      upload("lm_head.weight", base + o_head);
    } else {
      upload_q8("lm_head", 0, V, H, 0, 1);
      finish_q8(V, H, base + o_head, nullptr);
      // Stage images of each phase's rows of the head (the persistent kernel's head rows).
      for (int ph = 0; ph < 3; ++ph) {
        if (!qbase || qh_off[ph] == SIZE_MAX) continue;
        const PhaseRows pr = phase_rows(d, ph);
        launch_q_image(reinterpret_cast<const uint8_t *>(raw_q) + size_t(pr.row0) * H * bits / 8,
                       raw_s + size_t(pr.row0) * (H / 64), raw_b + size_t(pr.row0) * (H / 64), pr.n_main, H, bits,
                       qbase + qh_off[ph], st);
        m->qhead[ph] = qbase + qh_off[ph];
      }
      YAR_CUDA(cudaStreamSynchronize(st));
    }
    upload("model.norm.weight", base + o_norm);
    m->layers.resize(d.layers);
    for (int i = 0; i < d.layers; ++i) {
      const std::string n = "model.layers." + std::to_string(i), a = n + ".self_attn";
      if (bits) {  // one GPU (quantized weights are not built for tensor parallelism)
        upload_q8(a + ".q_proj", 0, Q, H, 0, 1);
        upload_q8(a + ".k_proj", 0, KV, H, Q, 1);
        upload_q8(a + ".v_proj", 0, KV, H, Q + KV, 1);
        auto img = [&](size_t o) { return qbase ? qbase + o : nullptr; };
        finish_q8(Q + 2 * KV, H, base + lo[i].qkv, img(qlo[i].qkv));
        upload_q8(a + ".o_proj", 0, H, Q, 0, 1);
        finish_q8(H, Q, base + lo[i].o, img(qlo[i].o));
        upload_q8(n + ".mlp.gate_proj", 0, F, H, 0, 2);
        upload_q8(n + ".mlp.up_proj", 0, F, H, 1, 2);
        finish_q8(2 * F, H, base + lo[i].gu, img(qlo[i].gu));
        upload_q8(n + ".mlp.down_proj", 0, H, F, 0, 1);
        finish_q8(H, F, base + lo[i].down, img(qlo[i].down));
        if (qbase) m->qlayers[i] = QLayer{img(qlo[i].qkv), img(qlo[i].o), img(qlo[i].gu), img(qlo[i].down)};
      } else {
      // Rank r: q rows of its heads, k/v rows of its KV heads, its FFN block of gate/up rows,
      // its hidden rows of O and down (all of them when tp_world == 1).
      upload_block(a + ".q_proj.weight", base + lo[i].qkv, plan.q_row0, Ql, 0, H);
      upload_block(a + ".k_proj.weight", base + lo[i].qkv + size_t(Ql) * H * e2, plan.kv_row0, KVl, 0, H);
      upload_block(a + ".v_proj.weight", base + lo[i].qkv + size_t(Ql + KVl) * H * e2, plan.kv_row0, KVl, 0, H);
      upload_block(a + ".o_proj.weight", base + lo[i].o, plan.h_row0, Hs, 0, Q);
      upload_gate_up(n + ".mlp.gate_proj.weight", n + ".mlp.up_proj.weight", base + lo[i].gu, plan.ffn_row0, Fl);
      upload_block(n + ".mlp.down_proj.weight", base + lo[i].down, plan.h_row0, Hs, 0, F);
      }
      upload(n + ".input_layernorm.weight", base + lo[i].ln1);
      upload(n + ".post_attention_layernorm.weight", base + lo[i].ln2);
      upload(a + ".q_norm.weight", base + lo[i].qn);
      upload(a + ".k_norm.weight", base + lo[i].kn);
      m->layers[i] = LayerWeights{at(lo[i].qkv), at(lo[i].o), at(lo[i].gu), at(lo[i].down),
                                  at(lo[i].ln1), at(lo[i].ln2), at(lo[i].qn), at(lo[i].kn)};
    }
    YAR_CUDA(cudaMalloc(&m->d_layers, sizeof(LayerWeights) * d.layers));
    YAR_CUDA(cudaMemcpy(m->d_layers, m->layers.data(), sizeof(LayerWeights) * d.layers, cudaMemcpyHostToDevice));
    if (!m->qlayers.empty()) {
      YAR_CUDA(cudaMalloc(&m->d_qlayers, sizeof(QLayer) * d.layers));
      YAR_CUDA(cudaMemcpy(m->d_qlayers, m->qlayers.data(), sizeof(QLayer) * d.layers, cudaMemcpyHostToDevice));
    }
    build_stage_maps(*m);
    m->embed = at(o_embed);
    m->lm_head = at(o_head);
    m->final_norm = at(o_norm);
    // RoPE tables (modeling_yue2.py:142-156): FP32 inv_freq = 1 / float(theta ** (2i/d)),
    // FP32 angle = pos * inv_freq, cos/sin evaluated in double, rounded to FP32, then
    // to BF16 (the activation dtype they are cast to before use).
    {
      const int half = D / 2;
      std::vector<float> inv(half), c(size_t(d.context) * half), s(size_t(d.context) * half);
      for (int i = 0; i < half; ++i) {
        const float e = f_div(float(2 * i), float(D));
        const float pw = float(std::pow(double(float(d.theta)), double(e)));
        inv[i] = f_div(1.0f, pw);
      }
      for (int pos = 0; pos < d.context; ++pos)
        for (int i = 0; i < half; ++i) {
          const float ang = f_mul(float(pos), inv[i]);
          c[size_t(pos) * half + i] = round_bf16(float(std::cos(double(ang))));
          s[size_t(pos) * half + i] = round_bf16(float(std::sin(double(ang))));
        }
      YAR_CUDA(cudaStreamSynchronize(st));
      YAR_CUDA(cudaMemcpy(base + o_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice));
      YAR_CUDA(cudaMemcpy(base + o_sin, s.data(), s.size() * 4, cudaMemcpyHostToDevice));
      m->rope_cos = reinterpret_cast<const float *>(base + o_cos);
      m->rope_sin = reinterpret_cast<const float *>(base + o_sin);
    }
    YAR_CUDA(cudaStreamSynchronize(st));
    YAR_CUDA(cudaEventDestroy(done[0]));
    YAR_CUDA(cudaEventDestroy(done[1]));
    YAR_CUDA(cudaStreamDestroy(st));
    YAR_CUDA(cudaFreeHost(stage));
    ::close(fd);
    if (tp_world > 1) tp_init(*m, tp_rank, tp_world, nccl_id);
  } catch (...) {
    tp_destroy(*m);
    if (m->arena) cudaFree(m->arena);
    if (m->d_layers) cudaFree(m->d_layers);
    if (m->d_wmaps) cudaFree(m->d_wmaps);
    if (m->qarena) cudaFree(m->qarena);
    if (m->d_qlayers) cudaFree(m->d_qlayers);
    delete m;
    throw;
  }
  return m;
}

void free_model(Model *m) {
  if (!m) return;
  cudaSetDevice(m->device);
  tp_destroy(*m);
  if (m->arena) cudaFree(m->arena);
  if (m->d_layers) cudaFree(m->d_layers);
  if (m->d_wmaps) cudaFree(m->d_wmaps);
  if (m->qarena) cudaFree(m->qarena);
  if (m->d_qlayers) cudaFree(m->d_qlayers);
  delete m;
}

}  // namespace yar
