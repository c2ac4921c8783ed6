// Qwen-Image quantized transformer: weights by GGUF name, device workspace, the forward
// pass over a batch of 1 or 2 sequences (conditional + unconditional CFG prompts) as a
// sequence of this library's kernels, and the denoising loop replayed from one captured
// CUDA graph per shape.
//
// Math order follows mold's quantized Qwen-Image transformer:
//   model forward        qwen_image/quantized_transformer.rs:1048-1139
//   block forward        qwen_image/quantized_transformer.rs:856-959
//   JointAttention       qwen_image/quantized_transformer.rs:695-816
//   OutputLayer          qwen_image/quantized_transformer.rs:962-989 (chunks: scale, shift)
//   RoPE positions       qwen_image/quantized_transformer.rs:339-435
//   step loop + CFG      qwen_image/pipeline.rs:2655-2716, scheduler sampling.rs:54-129
//
// A Qwen block has the structure of a FLUX double block (two streams, joint attention,
// GELU-tanh MLP, gate-residual updates), so it runs on the same kernels. What differs:
//  * to_q / to_k / to_v (and add_q/k/v_proj) are separate GGUF tensors; their raw rows
//    are concatenated once into one [3h, h] weight per stream (GGML blocks run along a
//    row, so row concatenation is a byte copy) and run as one GEMM.
//  * the text keys carry a mask. Attention does not depend on the order of its keys, so
//    the QK-norm/RoPE kernel writes the k / v of kept text keys first, then the image
//    keys, then the masked ones (kv_pos), and attention reads only the kept prefix.
//  * the text stem is RMSNorm(txt) -> txt_in, and the timestep MLP has no guidance or
//    pooled-text branch.
//
// HBM layout (B = batch, Lt / Li = text / image tokens, L = Lt + Li, h, m = mlp hidden):
//   x   f32  [B*Lt + B*Li, h]  residual stream: all text rows (batch-major), then all
//                              image rows, so each stream's linears are one GEMM over
//                              B*Lt or B*Li rows
//   xm  bf16 [same rows, h]    LayerNorm+modulate output
//   Y   bf16 [same rows, 3h+m] cols [0,3h) q|k|v, attention output over the v columns,
//                              [3h, 3h+m) GELU(mlp)
//   q,k,v bf16 [B][H][L][128]  per sequence: text positions 0..Lt, image Lt..L (k / v
//                              permuted by kv_pos)
//   pe  f32  [L, 64, 2, 2]     RoPE table shared by the batch
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "model_util.h"

using namespace mb;

struct mb_qwen {
  mb_qwen_config cfg;
  int device = 0;
  int64_t max_txt = 0, max_img = 0;
  int max_batch = 1;
  std::map<std::string, mb_weight*> mats;
  std::map<std::string, Vec1> vecs;
  bool finalized = false;

  // per block, fused q|k|v weights and biases: [0] text stream, [1] image stream
  std::vector<mb_weight*> qkv_w[2];
  std::vector<float*> qkv_b[2];

  // workspace
  float* x = nullptr;
  __nv_bfloat16* xm = nullptr;
  __nv_bfloat16* Y = nullptr;
  __nv_bfloat16 *q = nullptr, *k = nullptr, *v = nullptr;
  float* pe = nullptr;
  float* ids = nullptr;
  int* kv_pos = nullptr;
  __nv_bfloat16* txt_bf = nullptr;
  __nv_bfloat16* img_bf = nullptr;
  float* pred = nullptr;
  float* scal = nullptr;  // [0] t, [2] dt, [3] sigma_next, [4] 1 - sigma_next
  int* counter = nullptr;
  double* sched = nullptr;
  int sched_cap = 0;
  float t_scale = 1.f;     // temb argument = scal[0] * t_scale
  float* temb = nullptr;   // [256]
  float* hid = nullptr;    // [h]
  float* tvec = nullptr;   // [h]  timestep embedding
  float* mods = nullptr;
  float* gemv_stage = nullptr;
  std::vector<int64_t> mod_off;
  int64_t mod_off_final = 0;
  GemvJob* jobs_dev = nullptr;
  int gemv_kinds = 0;  // bit gemv_kind(type) of every GEMV job's weight type
  int64_t gemv_smem_rb = 0;  // largest row_bytes a GEMV block stages in shared memory
  int* blocks_dev = nullptr;
  int n_blocks[3] = {0, 0, 0}, block0[3] = {0, 0, 0};

  // per-call state from the mask
  std::vector<int64_t> n_valid;  // kept keys per sequence

  // graph cache
  cudaGraphExec_t graph = nullptr;
  std::vector<int64_t> graph_key;

  int64_t H() const { return cfg.num_heads; }
  int64_t h() const { return cfg.hidden_size; }
  int64_t mh() const { return cfg.mlp_hidden; }
  int64_t ldY() const { return 3 * h() + mh(); }
  int64_t rows() const { return (int64_t)max_batch * (max_txt + max_img); }
};

namespace {

struct Expected {
  std::string name;
  std::vector<int64_t> shape;
  bool required;
};

const char* kAttnLinears[8] = {"to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj", "to_out.0",
                               "to_add_out"};
const char* kNorms[4] = {"norm_q", "norm_k", "norm_added_q", "norm_added_k"};

std::vector<Expected> expected_tensors(const mb_qwen_config& c) {
  std::vector<Expected> out;
  const int64_t h = c.hidden_size, m = c.mlp_hidden, hd = h / c.num_heads;
  auto lin = [&](const std::string& n, int64_t o, int64_t i) {
    out.push_back({n + ".weight", {o, i}, true});
    out.push_back({n + ".bias", {o}, false});
  };
  lin("time_text_embed.timestep_embedder.linear_1", h, 256);
  lin("time_text_embed.timestep_embedder.linear_2", h, h);
  lin("img_in", h, c.in_channels);
  lin("txt_in", h, c.joint_attention_dim);
  out.push_back({"txt_norm.weight", {c.joint_attention_dim}, true});
  for (int i = 0; i < c.num_layers; i++) {
    const std::string p = "transformer_blocks." + std::to_string(i) + ".";
    for (const char* n : kAttnLinears) lin(p + "attn." + n, h, h);
    for (const char* n : kNorms) out.push_back({p + "attn." + n + ".weight", {hd}, true});
    for (const char* s : {"img", "txt"}) {
      const std::string S(s);
      lin(p + S + "_mlp.net.0.proj", m, h);
      lin(p + S + "_mlp.net.2", h, m);
      lin(p + S + "_mod.1", 6 * h, h);
    }
  }
  lin("norm_out.linear", 2 * h, h);
  lin("proj_out", (int64_t)c.patch_size * c.patch_size * c.out_channels, h);
  return out;
}

bool is_gemv_weight(const std::string& n) {
  return n.find("_mod.1.") != std::string::npos || n.rfind("norm_out.linear", 0) == 0 ||
         n.rfind("time_text_embed", 0) == 0;
}

const float* bias_or_null(const mb_qwen* m, const std::string& n) {
  auto it = m->vecs.find(n);
  return it == m->vecs.end() ? nullptr : it->second.dev;
}
const mb_weight* Wt(const mb_qwen* m, const std::string& n) { return m->mats.at(n); }
const float* Vt(const mb_qwen* m, const std::string& n) { return m->vecs.at(n).dev; }

std::string blk(int i) { return "transformer_blocks." + std::to_string(i) + "."; }

// Concatenates the rows of three [h, h] weights (same GGML type) into one [3h, h] weight.
mb_status fuse_rows(const mb_weight* a, const mb_weight* b, const mb_weight* c, mb_weight** out) {
  MB_CHECK(a->type == b->type && a->type == c->type && a->row_bytes == b->row_bytes && a->row_bytes == c->row_bytes &&
               a->n_cols == b->n_cols && a->n_cols == c->n_cols,
           MB_ERR_UNSUPPORTED, "q, k and v projections of a block must share one GGML type");
  mb_weight* w = new mb_weight(*a);
  w->n_rows = a->n_rows + b->n_rows + c->n_rows;
  const size_t sa = (size_t)a->n_rows * a->row_bytes, sb = (size_t)b->n_rows * b->row_bytes,
               sc = (size_t)c->n_rows * c->row_bytes;
  if (cudaMalloc(&w->dev, sa + sb + sc) != cudaSuccess) {
    delete w;
    return set_error(MB_ERR_NOMEM, "fused qkv alloc failed");
  }
  cudaError_t e = cudaMemcpy(w->dev, a->dev, sa, cudaMemcpyDeviceToDevice);
  if (e == cudaSuccess) e = cudaMemcpy((char*)w->dev + sa, b->dev, sb, cudaMemcpyDeviceToDevice);
  if (e == cudaSuccess) e = cudaMemcpy((char*)w->dev + sa + sb, c->dev, sc, cudaMemcpyDeviceToDevice);
  if (e != cudaSuccess) {
    mb_weight_destroy(w);
    return cuda_error(e, "fused qkv copy");
  }
  *out = w;
  return MB_OK;
}

mb_status fuse_bias(const mb_qwen* m, const std::string& p, const char* const* names, float** out) {
  const int64_t h = m->h();
  MB_TRY(dalloc(out, (size_t)(3 * h)));
  MB_CUDA(cudaMemset(*out, 0, 3 * h * sizeof(float)));
  for (int j = 0; j < 3; j++) {
    const float* b = bias_or_null(m, p + names[j] + ".bias");
    if (b) MB_CUDA(cudaMemcpy(*out + j * h, b, h * sizeof(float), cudaMemcpyDeviceToDevice));
  }
  return MB_OK;
}

mb_status finalize(mb_qwen* m) {
  const int64_t h = m->h();
  const mb_qwen_config& c = m->cfg;
  // ---- fused q|k|v per stream
  const char* txt_names[3] = {"add_q_proj", "add_k_proj", "add_v_proj"};
  const char* img_names[3] = {"to_q", "to_k", "to_v"};
  for (int i = 0; i < c.num_layers; i++) {
    const std::string p = blk(i) + "attn.";
    for (int s = 0; s < 2; s++) {
      const char* const* nm = s == 0 ? txt_names : img_names;
      mb_weight* w = nullptr;
      MB_TRY(fuse_rows(Wt(m, p + nm[0] + ".weight"), Wt(m, p + nm[1] + ".weight"), Wt(m, p + nm[2] + ".weight"), &w));
      m->qkv_w[s].push_back(w);
      float* b = nullptr;
      MB_TRY(fuse_bias(m, p, nm, &b));
      m->qkv_b[s].push_back(b);
      for (int j = 0; j < 3; j++) {
        const std::string n = p + nm[j] + ".weight";
        mb_weight_destroy(m->mats[n]);
        m->mats.erase(n);
      }
    }
  }
  // ---- GEMV job tables: [0] timestep linear_1, [1] linear_2, [2] all modulations
  std::vector<GemvJob> jobs;
  std::vector<int> blocks;
  auto add = [&](const std::string& name, float* y) {
    const mb_weight* w = Wt(m, name + ".weight");
    GemvJob j = {};
    j.w = w->dev;
    j.type = w->type;
    m->gemv_kinds |= 1 << gemv_kind(w->type);
    m->gemv_smem_rb = std::max(m->gemv_smem_rb, gemv_smem_row_bytes(w->type, w->row_bytes));
    j.n_rows = (int)w->n_rows;
    j.n_cols = (int)w->n_cols;
    j.row_bytes = w->row_bytes;
    j.bias = bias_or_null(m, name + ".bias");
    j.y = y;
    j.x_slot = 0;
    const int id = (int)jobs.size();
    jobs.push_back(j);
    for (int r = 0; r < j.n_rows; r += kGemvRowsPerBlock) {
      blocks.push_back(id);
      blocks.push_back(r);
    }
  };
  add("time_text_embed.timestep_embedder.linear_1", m->hid);
  m->n_blocks[0] = (int)blocks.size() / 2;
  m->block0[1] = m->n_blocks[0];
  add("time_text_embed.timestep_embedder.linear_2", m->tvec);
  m->n_blocks[1] = (int)blocks.size() / 2 - m->block0[1];
  m->block0[2] = m->block0[1] + m->n_blocks[1];
  int64_t off = 0;
  m->mod_off.clear();
  for (int i = 0; i < c.num_layers; i++) {
    m->mod_off.push_back(off);
    off += 12 * h;
  }
  m->mod_off_final = off;
  off += 2 * h;
  MB_TRY(dalloc(&m->mods, (size_t)off));
  for (int i = 0; i < c.num_layers; i++) {
    add(blk(i) + "img_mod.1", m->mods + m->mod_off[i]);
    add(blk(i) + "txt_mod.1", m->mods + m->mod_off[i] + 6 * h);
  }
  add("norm_out.linear", m->mods + m->mod_off_final);
  m->n_blocks[2] = (int)blocks.size() / 2 - m->block0[2];
  MB_TRY(dalloc(&m->jobs_dev, jobs.size()));
  MB_TRY(dalloc(&m->blocks_dev, blocks.size()));
  MB_CUDA(cudaMemcpy(m->jobs_dev, jobs.data(), jobs.size() * sizeof(GemvJob), cudaMemcpyHostToDevice));
  MB_CUDA(cudaMemcpy(m->blocks_dev, blocks.data(), blocks.size() * sizeof(int), cudaMemcpyHostToDevice));
  m->finalized = true;
  return MB_OK;
}

mb_status gemv_table(const mb_qwen* m, int table, const GemvInput* in, cudaStream_t st) {
  return check_launch(launch_gemv_batch(m->jobs_dev, m->gemv_kinds, m->blocks_dev + 2 * m->block0[table], m->n_blocks[table], in,
                                        1, m->gemv_stage, m->gemv_smem_rb, st),
                      "gemv batch");
}

mb_status gemm(const mb_weight* w, const float* bias, const void* x, int64_t M, int64_t ldx, void* y, int64_t ldy,
               bool out_bf16, int epi, const float* gate, const char* what, cudaStream_t st) {
  GemmEpilogue e;
  e.kind = epi;
  e.out_bf16 = out_bf16;
  e.gelu_from = epi == MB_EPI_GELU_TANH ? 0 : (int64_t)1 << 40;
  e.y = y;
  e.ldy = ldy;
  e.bias = bias;
  e.gate = gate;
  e.res = (const float*)y;
  e.ldr = ldy;
  if (g_prof) g_prof->begin(st);
  mb_status s = check_launch(launch_qgemm(w, x, M, ldx, e, st), what);
  if (g_prof) g_prof->end(st, std::string("gemm ") + what);
  return s;
}

// The text- and image-stream linears of a block as one grouped launch ([0] text, [1] image).
// With the gate-residual epilogue, y is also the residual.
mb_status gemm_pair(const mb_weight* const* w, const float* const* bias, const Seg* segs, const void* const* xs,
                    int64_t ldx, void* const* ys, int64_t ldy, bool out_bf16, int epi, const float* const* gates,
                    const char* what, cudaStream_t st) {
  GemmProblem g[2];
  for (int s = 0; s < 2; s++) {
    GemmEpilogue& e = g[s].epi;
    e.kind = epi;
    e.out_bf16 = out_bf16;
    e.gelu_from = epi == MB_EPI_GELU_TANH ? 0 : (int64_t)1 << 40;
    e.y = ys[s];
    e.ldy = ldy;
    e.bias = bias[s];
    e.gate = gates ? gates[s] : nullptr;
    e.res = (const float*)ys[s];
    e.ldr = ldy;
    g[s].w = w[s];
    g[s].x = xs[s];
    g[s].M = segs[s].rows;
    g[s].ldx = ldx;
  }
  const bool same = w[0]->type == w[1]->type;
  if (g_prof) g_prof->begin(st);
  mb_status r = MB_OK;
  if (same) {
    r = check_launch(launch_qgemm_group(2, g, st), what);
  } else {  // the grouped kernel is instantiated per weight type
    for (int s = 0; s < 2 && r == MB_OK; s++) r = check_launch(launch_qgemm_group(1, &g[s], st), what);
  }
  if (g_prof) g_prof->end(st, std::string("gemm txt+img ") + what);
  return r;
}

// Forward over B sequences. img: f32 latents, sequence b at img + b * img_stride (stride 0:
// every sequence denoises the same latent, as in the CFG batch); txt f32 [B*Lt, jad].
// t (scal[0]) is read on the device.
mb_status run_forward(mb_qwen* m, const float* img, int64_t img_stride, int64_t Li, const float* txt, int64_t Lt,
                      int B, cudaStream_t st) {
  const mb_qwen_config& c = m->cfg;
  const int64_t h = m->h(), H = m->H(), L = Lt + Li, ldY = m->ldY();
  const int64_t Rt = (int64_t)B * Lt, Ri = (int64_t)B * Li;
  const int cin = c.in_channels;
  // ---- timestep MLP and every modulation vector
  TIMED("timestep_embedding",
        check_launch(launch_timestep_embedding(m->scal, m->t_scale, m->temb, 256, st), "timestep embedding"));
  {
    GemvInput in = {};
    in.parts[0] = m->temb;
    in.n_parts = 1;
    in.len = 256;
    TIMED("gemv timestep", gemv_table(m, 0, &in, st));
    in.len = (int)h;
    in.parts[0] = m->hid;
    in.apply_silu = 1;
    TIMED("gemv timestep", gemv_table(m, 1, &in, st));
    in.parts[0] = m->tvec;
    TIMED("gemv modulations", gemv_table(m, 2, &in, st));
  }
  // ---- stems: txt_in(RMSNorm(txt)) into the text rows, img_in(img) into the image rows
  TIMED("rms_norm", check_launch(launch_rms_norm(txt, Rt, c.joint_attention_dim, c.joint_attention_dim,
                                                 Vt(m, "txt_norm.weight"), 1e-6f, m->txt_bf, c.joint_attention_dim, st),
                                 "txt_norm"));
  MB_TRY(gemm(Wt(m, "txt_in.weight"), bias_or_null(m, "txt_in.bias"), m->txt_bf, Rt, c.joint_attention_dim, m->x, h,
              false, MB_EPI_NONE, nullptr, "txt_in", st));
  for (int b = 0; b < B; b++)
    TIMED("cast_f32_bf16", check_launch(launch_cast_f32_bf16(img + b * img_stride, Li, cin, cin,
                                                             m->img_bf + (int64_t)b * Li * cin, cin, st),
                                        "cast img"));
  MB_TRY(gemm(Wt(m, "img_in.weight"), bias_or_null(m, "img_in.bias"), m->img_bf, Ri, cin, m->x + Rt * h, h, false,
              MB_EPI_NONE, nullptr, "img_in", st));

  const Seg segs[2] = {{0, Rt}, {Rt, Ri}};  // text, image
  const int64_t qkv_stride = H * L * 128;  // one sequence in q / k / v
  for (int i = 0; i < c.num_layers; i++) {
    const std::string p = blk(i);
    const float* mos[2] = {m->mods + m->mod_off[i] + 6 * h, m->mods + m->mod_off[i]};  // txt_mod, img_mod
    {
      LnSegs ls = {};
      ls.n = 2;
      for (int s = 0; s < 2; s++) ls.s[s] = {segs[s].row0, segs[s].rows, mos[s], mos[s] + h};
      TIMED("ln_modulate", check_launch(launch_ln_modulate_segs(m->x, h, h, ls, m->xm, h, st), "ln_mod1"));
    }
    {
      const mb_weight* w[2] = {m->qkv_w[0][i], m->qkv_w[1][i]};
      const float* bs[2] = {m->qkv_b[0][i], m->qkv_b[1][i]};
      const void* xs[2] = {m->xm, m->xm + Rt * h};
      void* ys[2] = {m->Y, m->Y + Rt * ldY};
      MB_TRY(gemm_pair(w, bs, segs, xs, h, ys, ldY, true, MB_EPI_NONE, nullptr, "qkv", st));
    }
    {
      QkSegs qs = {};
      for (int b = 0; b < B; b++) {
        for (int s = 0; s < 2; s++) {  // text, image rows of sequence b
          QkSeg& g = qs.s[qs.n++];
          g.row0 = s == 0 ? (int64_t)b * Lt : Rt + (int64_t)b * Li;
          g.rows = s == 0 ? Lt : Li;
          g.pos0 = s == 0 ? 0 : Lt;
          g.off = b * qkv_stride;
          g.kv_pos = m->kv_pos + (int64_t)b * L;
          g.qs = Vt(m, p + (s == 0 ? "attn.norm_added_q.weight" : "attn.norm_q.weight"));
          g.ks = Vt(m, p + (s == 0 ? "attn.norm_added_k.weight" : "attn.norm_k.weight"));
        }
      }
      TIMED("qk_norm_rope", check_launch(launch_qk_norm_rope_segs(m->Y, ldY, (int)H, m->pe, L, qs, m->q, m->k, m->v, st),
                                         "qk_norm_rope"));
    }
    for (int b = 0; b < B; b++) {
      const int64_t o = b * qkv_stride;
      TIMED("attention", check_launch(launch_attention(m->q + o, m->k + o, m->v + o, (int)H, L, L, m->n_valid[b],
                                                       m->Y + (int64_t)b * Lt * ldY + 2 * h, ldY, st, Lt,
                                                       m->Y + (Rt + (int64_t)b * Li) * ldY + 2 * h),
                                      "attention"));
    }
    {
      const mb_weight* w[2] = {Wt(m, p + "attn.to_add_out.weight"), Wt(m, p + "attn.to_out.0.weight")};
      const float* bs[2] = {bias_or_null(m, p + "attn.to_add_out.bias"), bias_or_null(m, p + "attn.to_out.0.bias")};
      const void* xs[2] = {m->Y + 2 * h, m->Y + Rt * ldY + 2 * h};
      void* ys[2] = {m->x, m->x + Rt * h};
      const float* gates[2] = {mos[0] + 2 * h, mos[1] + 2 * h};
      MB_TRY(gemm_pair(w, bs, segs, xs, ldY, ys, h, false, MB_EPI_GATE_RESIDUAL, gates, "attn out", st));
    }
    {
      LnSegs ls = {};
      ls.n = 2;
      for (int s = 0; s < 2; s++) ls.s[s] = {segs[s].row0, segs[s].rows, mos[s] + 3 * h, mos[s] + 4 * h};
      TIMED("ln_modulate", check_launch(launch_ln_modulate_segs(m->x, h, h, ls, m->xm, h, st), "ln_mod2"));
    }
    {
      const mb_weight* w[2] = {Wt(m, p + "txt_mlp.net.0.proj.weight"), Wt(m, p + "img_mlp.net.0.proj.weight")};
      const float* bs[2] = {bias_or_null(m, p + "txt_mlp.net.0.proj.bias"),
                            bias_or_null(m, p + "img_mlp.net.0.proj.bias")};
      const void* xs[2] = {m->xm, m->xm + Rt * h};
      void* ys[2] = {m->Y + 3 * h, m->Y + Rt * ldY + 3 * h};
      MB_TRY(gemm_pair(w, bs, segs, xs, h, ys, ldY, true, MB_EPI_GELU_TANH, nullptr, "mlp.0", st));
    }
    {
      const mb_weight* w[2] = {Wt(m, p + "txt_mlp.net.2.weight"), Wt(m, p + "img_mlp.net.2.weight")};
      const float* bs[2] = {bias_or_null(m, p + "txt_mlp.net.2.bias"), bias_or_null(m, p + "img_mlp.net.2.bias")};
      const void* xs[2] = {m->Y + 3 * h, m->Y + Rt * ldY + 3 * h};
      void* ys[2] = {m->x, m->x + Rt * h};
      const float* gates[2] = {mos[0] + 5 * h, mos[1] + 5 * h};
      MB_TRY(gemm_pair(w, bs, segs, xs, ldY, ys, h, false, MB_EPI_GATE_RESIDUAL, gates, "mlp.2", st));
    }
  }
  // ---- output layer on the image rows: LN * (1 + scale) + shift, scale first
  {
    const float* mo = m->mods + m->mod_off_final;
    TIMED("ln_modulate", check_launch(launch_ln_modulate(m->x + Rt * h, Ri, h, h, mo + h, mo, m->xm + Rt * h, h, st),
                                      "ln_final"));
    MB_TRY(gemm(Wt(m, "proj_out.weight"), bias_or_null(m, "proj_out.bias"), m->xm + Rt * h, Ri, h, m->pred, cin,
                false, MB_EPI_NONE, nullptr, "proj_out", st));
  }
  return MB_OK;
}

mb_status check_complete(const mb_qwen* m) {
  if (m->finalized) return MB_OK;
  for (const auto& e : expected_tensors(m->cfg)) {
    if (!e.required) continue;
    const bool have = e.shape.size() == 1 ? m->vecs.count(e.name) > 0 : m->mats.count(e.name) > 0;
    MB_CHECK(have, MB_ERR_NOT_READY, "Qwen-Image model is missing tensor " + e.name);
  }
  return MB_OK;
}

// RoPE table, key order and kept-key counts for this call's shapes and mask.
mb_status prepare(mb_qwen* m, int64_t h_tok, int64_t w_tok, const uint8_t* mask, int64_t Lt, int B,
                  cudaStream_t st) {
  MB_TRY(check_complete(m));
  if (!m->finalized) MB_TRY(finalize(m));
  const int64_t Li = h_tok * w_tok, L = Lt + Li;
  MB_CHECK(h_tok >= 1 && w_tok >= 1 && Lt >= 1 && Lt <= m->max_txt && Li <= m->max_img, MB_ERR_INVALID,
           "sequence lengths exceed the model's workspace (max_txt / max_img)");
  MB_CHECK(B >= 1 && B <= m->max_batch, MB_ERR_INVALID, "batch exceeds the model's max_batch");
  // positions (QwenRopeEmbedder::forward with frame = 1): text rows first
  std::vector<float> ids((size_t)L * 3);
  const int64_t s0 = (h_tok / 2 > w_tok / 2) ? h_tok / 2 : w_tok / 2;
  for (int64_t i = 0; i < Lt; i++) ids[i * 3] = ids[i * 3 + 1] = ids[i * 3 + 2] = (float)(s0 + i);
  const int64_t hn = h_tok - h_tok / 2, wn = w_tok - w_tok / 2;
  for (int64_t y = 0; y < h_tok; y++)
    for (int64_t xx = 0; xx < w_tok; xx++) {
      float* r = &ids[(Lt + y * w_tok + xx) * 3];
      r[0] = 0.f;
      r[1] = (float)(y - hn);
      r[2] = (float)(xx - wn);
    }
  // key order: kept text keys, image keys, masked text keys
  std::vector<uint8_t> hm((size_t)B * Lt, 1);
  if (mask) MB_CUDA(cudaMemcpy(hm.data(), mask, hm.size(), cudaMemcpyDeviceToHost));
  std::vector<int> pos((size_t)B * L);
  m->n_valid.assign(B, 0);
  for (int b = 0; b < B; b++) {
    const uint8_t* mb = &hm[(size_t)b * Lt];
    int64_t nv = 0;
    for (int64_t i = 0; i < Lt; i++) nv += mb[i] != 0;
    int64_t kept = 0, dropped = 0;
    int* pb = &pos[(size_t)b * L];
    for (int64_t i = 0; i < Lt; i++) pb[i] = mb[i] ? (int)kept++ : (int)(nv + Li + dropped++);
    for (int64_t j = 0; j < Li; j++) pb[Lt + j] = (int)(nv + j);
    m->n_valid[b] = nv + Li;
  }
  MB_CUDA(cudaMemcpyAsync(m->ids, ids.data(), ids.size() * sizeof(float), cudaMemcpyHostToDevice, st));
  MB_CUDA(cudaMemcpyAsync(m->kv_pos, pos.data(), pos.size() * sizeof(int), cudaMemcpyHostToDevice, st));
  MB_CUDA(launch_rope_table(m->ids, L, 3, m->cfg.axes_dim, m->cfg.theta, m->pe, st));
  // the host vectors die here: finish the copies first
  MB_CUDA(cudaStreamSynchronize(st));
  return MB_OK;
}

}  // namespace

extern "C" {

mb_status mb_qwen_create(const mb_qwen_config* cfg, int64_t max_txt, int64_t max_img, int max_batch, mb_qwen** out) {
  MB_CHECK(cfg && out, MB_ERR_INVALID, "NULL argument");
  *out = nullptr;
  MB_CHECK(cfg->num_heads > 0 && cfg->hidden_size == cfg->num_heads * 128, MB_ERR_UNSUPPORTED,
           "head_dim must be 128 (hidden_size == 128 * num_heads)");
  MB_CHECK(cfg->axes_dim[0] + cfg->axes_dim[1] + cfg->axes_dim[2] == 128 && cfg->axes_dim[0] % 2 == 0 &&
               cfg->axes_dim[1] % 2 == 0 && cfg->axes_dim[2] % 2 == 0,
           MB_ERR_INVALID, "axes_dim must be even and sum to 128");
  MB_CHECK(cfg->hidden_size % 256 == 0 && cfg->mlp_hidden % 256 == 0 && cfg->hidden_size <= 4096, MB_ERR_INVALID,
           "hidden and mlp sizes must be multiples of 256 (hidden <= 4096)");
  MB_CHECK(cfg->joint_attention_dim % 128 == 0 && cfg->joint_attention_dim <= 8192 && cfg->in_channels % 64 == 0 &&
               cfg->patch_size > 0 && cfg->in_channels == cfg->out_channels * cfg->patch_size * cfg->patch_size,
           MB_ERR_INVALID, "unsupported stem sizes");
  MB_CHECK(cfg->num_layers >= 0, MB_ERR_INVALID, "num_layers must be >= 0");
  MB_CHECK(max_txt > 0 && max_img > 0 && max_batch >= 1 && max_batch <= 2, MB_ERR_INVALID,
           "max_txt, max_img must be positive and max_batch 1 or 2");
  mb_qwen* m = new mb_qwen();
  m->cfg = *cfg;
  cudaGetDevice(&m->device);
  m->max_txt = max_txt;
  m->max_img = max_img;
  m->max_batch = max_batch;
  const int64_t R = m->rows(), L = max_txt + max_img, h = m->h(), H = m->H();
  mb_status s = MB_OK;
  if ((s = dalloc(&m->x, R * h)) || (s = dalloc(&m->xm, R * h)) || (s = dalloc(&m->Y, R * m->ldY())) ||
      (s = dalloc(&m->q, max_batch * H * L * 128)) || (s = dalloc(&m->k, max_batch * H * L * 128)) ||
      (s = dalloc(&m->v, max_batch * H * L * 128)) || (s = dalloc(&m->pe, L * 256)) || (s = dalloc(&m->ids, L * 3)) ||
      (s = dalloc(&m->kv_pos, max_batch * L)) ||
      (s = dalloc(&m->txt_bf, max_batch * max_txt * cfg->joint_attention_dim)) ||
      (s = dalloc(&m->img_bf, max_batch * max_img * cfg->in_channels)) ||
      (s = dalloc(&m->pred, max_batch * max_img * cfg->in_channels)) || (s = dalloc(&m->scal, 8)) ||
      (s = dalloc(&m->counter, 1)) || (s = dalloc(&m->temb, 256)) || (s = dalloc(&m->hid, h)) ||
      (s = dalloc(&m->tvec, h)) || (s = dalloc(&m->gemv_stage, gemv_stage_floats()))) {
    mb_qwen_destroy(m);
    return s;
  }
  *out = m;
  return MB_OK;
}

mb_status mb_qwen_destroy(mb_qwen* m) {
  if (!m) return MB_OK;
  if (m->graph) cudaGraphExecDestroy(m->graph);
  for (auto& kv : m->mats) mb_weight_destroy(kv.second);
  for (auto& kv : m->vecs) cudaFree(kv.second.dev);
  for (int s = 0; s < 2; s++) {
    for (mb_weight* w : m->qkv_w[s]) mb_weight_destroy(w);
    for (float* b : m->qkv_b[s]) cudaFree(b);
  }
  void* bufs[] = {m->x,       m->xm,    m->Y,   m->q,    m->k,    m->v,     m->pe,   m->ids,
                  m->kv_pos,  m->txt_bf, m->img_bf, m->pred, m->scal, m->counter, m->sched, m->temb,
                  m->hid,     m->tvec,  m->mods, m->jobs_dev, m->blocks_dev, m->gemv_stage};
  for (void* b : bufs)
    if (b) cudaFree(b);
  delete m;
  return MB_OK;
}

mb_status mb_qwen_set_tensor(mb_qwen* m, const char* name, int ggml_type, int64_t n_rows, int64_t n_cols,
                             const void* data, size_t nbytes, int data_on_device) {
  MB_CHECK(m && name && data, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(!m->finalized, MB_ERR_INVALID, "tensors cannot be replaced after the first forward");
  const std::string n(name);
  const std::vector<int64_t>* shape = nullptr;
  const auto exp = expected_tensors(m->cfg);
  for (const auto& e : exp)
    if (e.name == n) shape = &e.shape;
  MB_CHECK(shape, MB_ERR_INVALID, "unknown Qwen-Image tensor name '" + n + "'");
  if (shape->size() == 1) {
    MB_CHECK(n_rows * n_cols == (*shape)[0], MB_ERR_INVALID, "tensor '" + n + "' has the wrong length");
    Vec1 v;
    MB_TRY(upload_vec1(ggml_type, (*shape)[0], data, nbytes, data_on_device, &v));
    auto it = m->vecs.find(n);
    if (it != m->vecs.end()) cudaFree(it->second.dev);
    m->vecs[n] = v;
    return MB_OK;
  }
  MB_CHECK(n_rows == (*shape)[0] && n_cols == (*shape)[1], MB_ERR_INVALID,
           "tensor '" + n + "' has shape [" + std::to_string(n_rows) + ", " + std::to_string(n_cols) + "], expected [" +
               std::to_string((*shape)[0]) + ", " + std::to_string((*shape)[1]) + "]");
  mb_weight* w = nullptr;
  MB_TRY(upload_matrix(ggml_type, n_rows, n_cols, data, nbytes, data_on_device, !is_gemv_weight(n), &w));
  auto it = m->mats.find(n);
  if (it != m->mats.end()) mb_weight_destroy(it->second);
  m->mats[n] = w;
  return MB_OK;
}

mb_status mb_qwen_missing(const mb_qwen* m, char* buf, size_t buflen) {
  MB_CHECK(m && buf && buflen > 0, MB_ERR_INVALID, "NULL argument");
  std::string s;
  if (!m->finalized) {
    for (const auto& e : expected_tensors(m->cfg)) {
      if (!e.required) continue;
      const bool have = e.shape.size() == 1 ? m->vecs.count(e.name) > 0 : m->mats.count(e.name) > 0;
      if (!have) s += e.name + "\n";
    }
  }
  const size_t n = s.size() < buflen - 1 ? s.size() : buflen - 1;
  memcpy(buf, s.data(), n);
  buf[n] = 0;
  return MB_OK;
}

mb_status mb_qwen_forward(mb_qwen* m, const float* img, int64_t h_tokens, int64_t w_tokens, const float* txt,
                          const uint8_t* txt_mask, int64_t L_txt, int batch, float t, float* pred, void* stream) {
  MB_CHECK(m && img && txt && pred, MB_ERR_INVALID, "NULL argument");
  cudaStream_t st = (cudaStream_t)stream;
  MB_TRY(prepare(m, h_tokens, w_tokens, txt_mask, L_txt, batch, st));
  const int64_t Li = h_tokens * w_tokens;
  m->t_scale = 1.f;
  MB_CUDA(launch_set_scalars(m->scal, t, 0.f, st));
  OpProfiler prof;
  if (profile_requested()) g_prof = &prof;
  mb_status fs = run_forward(m, img, Li * m->cfg.in_channels, Li, txt, L_txt, batch, st);
  if (g_prof) {
    g_prof = nullptr;
    prof.report();
  }
  MB_TRY(fs);
  MB_CUDA(cudaMemcpyAsync(pred, m->pred, (size_t)batch * Li * m->cfg.in_channels * sizeof(float),
                          cudaMemcpyDeviceToDevice, st));
  return MB_OK;
}

mb_status mb_qwen_denoise_ex(mb_qwen* m, float* img, int64_t h_tokens, int64_t w_tokens, const float* txt,
                             const uint8_t* txt_mask, int64_t L_txt, int batch, const double* sigmas, int n_sigmas,
                             float guidance, const mb_inpaint* inpaint, mb_step_callback on_step, void* user,
                             void* stream) {
  MB_CHECK(m && img && txt && sigmas, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(!inpaint || (inpaint->mask && inpaint->original && inpaint->noise), MB_ERR_INVALID,
           "inpaint needs mask, original and noise");
  MB_CHECK(n_sigmas >= 2, MB_ERR_INVALID, "need at least two sigmas");
  cudaStream_t st = (cudaStream_t)stream;
  MB_TRY(prepare(m, h_tokens, w_tokens, txt_mask, L_txt, batch, st));
  const int64_t Li = h_tokens * w_tokens;
  const int cin = m->cfg.in_channels;
  if (m->sched_cap < n_sigmas) {
    if (m->sched) cudaFree(m->sched);
    m->sched = nullptr;
    const int cap = n_sigmas > 1024 ? n_sigmas : 1024;  // keeps the pointer (and the graph) stable
    MB_TRY(dalloc(&m->sched, (size_t)cap));
    m->sched_cap = cap;
  }
  MB_CUDA(cudaMemcpyAsync(m->sched, sigmas, n_sigmas * sizeof(double), cudaMemcpyHostToDevice, st));
  MB_CUDA(cudaMemsetAsync(m->counter, 0, sizeof(int), st));
  m->t_scale = 1000.f;  // QwenImageScheduler::current_timestep = sigma * 1000
  int32_t gbits;
  memcpy(&gbits, &guidance, sizeof(gbits));
  std::vector<int64_t> key = {(int64_t)(uintptr_t)img, (int64_t)(uintptr_t)txt, (int64_t)(uintptr_t)m->sched,
                              L_txt, Li, batch, (int64_t)gbits};
  for (int64_t nv : m->n_valid) key.push_back(nv);
  for (const void* p : {inpaint ? (const void*)inpaint->mask : nullptr, inpaint ? (const void*)inpaint->original : nullptr,
                        inpaint ? (const void*)inpaint->noise : nullptr})
    key.push_back((int64_t)(uintptr_t)p);
  const bool reuse = m->graph && key == m->graph_key;
  auto step_tail = [&](cudaStream_t s) -> cudaError_t {
    cudaError_t e;
    if (batch == 2)
      e = launch_cfg_euler(img, m->pred, m->pred + Li * cin, Li, m->cfg.out_channels,
                           m->cfg.patch_size * m->cfg.patch_size, guidance, 0.f, m->scal + 2, s);
    else
      e = launch_euler_dev(img, m->pred, Li * cin, m->scal + 2, s);
    if (e == cudaSuccess && inpaint)
      e = launch_inpaint_blend(img, Li * cin, m->scal, inpaint->mask, inpaint->original, inpaint->noise, s);
    return e;
  };
  if (!reuse) {
    if (m->graph) {
      cudaGraphExecDestroy(m->graph);
      m->graph = nullptr;
    }
    // Eager warm-up of one step's forward so every kernel attribute is set before capture.
    MB_CUDA(launch_step_prologue(m->sched, m->counter, m->scal, st));
    MB_TRY(run_forward(m, img, 0, Li, txt, L_txt, batch, st));
    MB_CUDA(cudaMemsetAsync(m->counter, 0, sizeof(int), st));
    MB_CUDA(cudaStreamSynchronize(st));
    cudaStream_t cs;
    MB_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    cudaGraph_t g;
    MB_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    cudaError_t pe = launch_step_prologue(m->sched, m->counter, m->scal, cs);
    mb_status s = run_forward(m, img, 0, Li, txt, L_txt, batch, cs);
    cudaError_t le = step_tail(cs);
    cudaError_t ce = cudaStreamEndCapture(cs, &g);
    cudaStreamDestroy(cs);
    if (s != MB_OK) return s;
    MB_CUDA(pe);
    MB_CUDA(le);
    MB_CUDA(ce);
    cudaError_t ie = cudaGraphInstantiate(&m->graph, g, 0);
    cudaGraphDestroy(g);
    MB_CUDA(ie);
    m->graph_key = key;
  }
  MB_CUDA(enqueue_steps(m->graph, n_sigmas - 1, on_step, user, st));
  return MB_OK;
}

mb_status mb_qwen_denoise(mb_qwen* m, float* img, int64_t h_tokens, int64_t w_tokens, const float* txt,
                          const uint8_t* txt_mask, int64_t L_txt, int batch, const double* sigmas, int n_sigmas,
                          float guidance, void* stream) {
  return mb_qwen_denoise_ex(m, img, h_tokens, w_tokens, txt, txt_mask, L_txt, batch, sigmas, n_sigmas, guidance,
                            nullptr, nullptr, nullptr, stream);
}

}  // extern "C"
