// FLUX.1 quantized transformer: weights by GGUF name, device workspace, the
// forward pass as a sequence of this library's kernels, and the denoising loop
// replayed from one captured CUDA graph per step shape.
//
// Math order follows mold's in-repo restatement of candle's FLUX model:
//   forward            flux/offload.rs:525-580
//   DoubleBlock        flux/offload.rs:275-323
//   SingleBlock        flux/offload.rs:377-396
//   FinalLayer         flux/offload.rs:421-429
//   denoise loop       flux/transformer.rs:50-95 (img += pred * (t_prev - t_curr))
//
// HBM layout of the activations (L = L_txt + L_img, h = hidden, m = mlp hidden):
//   x   f32  [L, h]         residual stream; txt rows 0..L_txt-1, then img rows, so the
//                           single-stream input cat[txt, img] is x itself (no concat copy)
//   xm  bf16 [L, h]         LayerNorm+modulate output = A operand of the next linear
//   Y   bf16 [L, 3h + m]    cols [0,3h): fused qkv / linear1 qkv part; the attention output
//                           is written over the consumed v columns [2h,3h); cols [3h, 3h+m):
//                           GELU(mlp) -> so [2h, 3h+m) is exactly cat[attn, gelu(mlp)], the
//                           input of single-block linear2 (and [3h, 3h+m) of double-block mlp.2)
//   q,k,v bf16 [H, L, 128]  attention layout written by the fused QK-norm/RoPE kernel
//   pe  f32  [L, 64, 2, 2]  RoPE table (computed once per denoise call)
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "model_util.h"

namespace mb {
cudaError_t launch_gemv_single(const mb_weight* w, const float* x, int apply_silu, const float* bias, float* y,
                               cudaStream_t st);
}

using namespace mb;

struct mb_flux {
  mb_flux_config cfg;
  int device = 0;
  int64_t max_txt = 0, max_img = 0;
  std::map<std::string, mb_weight*> mats;
  std::map<std::string, Vec1> vecs;
  bool finalized = false;

  // workspace
  float* x = nullptr;
  __nv_bfloat16* xm = nullptr;
  __nv_bfloat16* Y = nullptr;
  __nv_bfloat16 *q = nullptr, *k = nullptr, *v = nullptr;
  float* pe = nullptr;
  float* ids = nullptr;
  __nv_bfloat16* txt_bf = nullptr;
  __nv_bfloat16* img_bf = nullptr;
  float* pred = nullptr;
  float* scal = nullptr;   // [0] t, [1] guidance, [2] dt, [3] t_next, [4] 1 - t_next
  int* counter = nullptr;
  double* sched = nullptr;
  int sched_cap = 0;
  float* temb = nullptr;   // [2][256]
  float* hid = nullptr;    // [3][h]
  float* parts = nullptr;  // [3][h]
  float* mods = nullptr;   // all modulation vectors
  float* gemv_stage = nullptr;
  std::vector<int64_t> mod_off_double, mod_off_single;
  int64_t mod_off_final = 0, mod_total = 0;
  GemvJob* jobs_dev = nullptr;
  int gemv_kinds = 0;  // bit gemv_kind(type) of every GEMV job's weight type
  int64_t gemv_smem_rb = 0;  // largest row_bytes a GEMV block stages in shared memory
  int* blocks_dev = nullptr;
  int n_jobs[3] = {0, 0, 0}, n_blocks[3] = {0, 0, 0}, job0[3] = {0, 0, 0}, block0[3] = {0, 0, 0};

  // graph cache
  cudaGraphExec_t graph = nullptr;
  int64_t graph_lt = -1, graph_li = -1;
  const void* graph_key[7] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};

  int64_t H() const { return cfg.num_heads; }
  int64_t h() const { return cfg.hidden_size; }
  int64_t mh() const { return cfg.mlp_hidden; }
  int64_t ldY() const { return 3 * h() + mh(); }
};

namespace {

std::vector<std::pair<std::string, std::vector<int64_t>>> expected_tensors(const mb_flux_config& c) {
  std::vector<std::pair<std::string, std::vector<int64_t>>> out;
  const int64_t h = c.hidden_size, m = c.mlp_hidden, hd = h / c.num_heads;
  auto lin = [&](const std::string& n, int64_t o, int64_t i) {
    out.push_back({n + ".weight", {o, i}});
    out.push_back({n + ".bias", {o}});
  };
  lin("img_in", h, c.in_channels);
  lin("txt_in", h, c.context_in_dim);
  lin("time_in.in_layer", h, 256);
  lin("time_in.out_layer", h, h);
  lin("vector_in.in_layer", h, c.vec_in_dim);
  lin("vector_in.out_layer", h, h);
  if (c.guidance_embed) {
    lin("guidance_in.in_layer", h, 256);
    lin("guidance_in.out_layer", h, h);
  }
  for (int i = 0; i < c.depth; i++) {
    const std::string p = "double_blocks." + std::to_string(i) + ".";
    for (const char* s : {"img", "txt"}) {
      const std::string S(s);
      lin(p + S + "_mod.lin", 6 * h, h);
      lin(p + S + "_attn.qkv", 3 * h, h);
      out.push_back({p + S + "_attn.norm.query_norm.scale", {hd}});
      out.push_back({p + S + "_attn.norm.key_norm.scale", {hd}});
      lin(p + S + "_attn.proj", h, h);
      lin(p + S + "_mlp.0", m, h);
      lin(p + S + "_mlp.2", h, m);
    }
  }
  for (int i = 0; i < c.depth_single; i++) {
    const std::string p = "single_blocks." + std::to_string(i) + ".";
    lin(p + "linear1", 3 * h + m, h);
    lin(p + "linear2", h, h + m);
    out.push_back({p + "norm.query_norm.scale", {hd}});
    out.push_back({p + "norm.key_norm.scale", {hd}});
    lin(p + "modulation.lin", 3 * h, h);
  }
  lin("final_layer.linear", c.in_channels, h);
  lin("final_layer.adaLN_modulation.1", 2 * h, h);
  return out;
}

const mb_weight* W(const mb_flux* m, const std::string& n) { return m->mats.at(n); }
const float* B(const mb_flux* m, const std::string& n) { return m->vecs.at(n).dev; }

mb_status linear(const mb_flux* m, const std::string& name, const void* x, int64_t M, int64_t ldx, void* y,
                 int64_t ldy, bool out_bf16, int epi, int64_t gelu_from, const float* gate, cudaStream_t st) {
  GemmEpilogue e;
  e.kind = epi;
  e.out_bf16 = out_bf16;
  e.gelu_from = epi == MB_EPI_GELU_TANH ? gelu_from : (int64_t)1 << 40;
  e.y = y;
  e.ldy = ldy;
  e.bias = B(m, name + ".bias");
  e.gate = gate;
  e.res = (const float*)y;
  e.ldr = ldy;
  if (g_prof) g_prof->begin(st);
  mb_status s = check_launch(launch_qgemm(W(m, name + ".weight"), x, M, ldx, e, st), name.c_str());
  if (g_prof) {
    std::string role = name;
    const size_t d = role.find("blocks.");
    if (d != std::string::npos) role = role.substr(role.find('.', d + 7) + 1);
    g_prof->end(st, "gemm " + role + " M=" + std::to_string(M));
  }
  return s;
}

// The text- and image-stream linears of a double block ("<p>txt<suffix>", "<p>img<suffix>")
// as one grouped GEMM launch. For the gate-residual epilogue y is also the residual.
mb_status linear_pair(const mb_flux* m, const std::string& p, const char* suffix, const Seg* segs,
                      const void* const* xs, int64_t ldx, void* const* ys, int64_t ldy, bool out_bf16, int epi,
                      const float* const* gates, cudaStream_t st) {
  GemmProblem g[2];
  const char* S[2] = {"txt", "img"};
  for (int s = 0; s < 2; s++) {
    const std::string name = p + S[s] + suffix;
    GemmEpilogue& e = g[s].epi;
    e.kind = epi;
    e.out_bf16 = out_bf16;
    e.gelu_from = epi == MB_EPI_GELU_TANH ? 0 : (int64_t)1 << 40;
    e.y = ys[s];
    e.ldy = ldy;
    e.bias = B(m, name + ".bias");
    e.gate = gates[s];
    e.res = (const float*)ys[s];
    e.ldr = ldy;
    g[s].w = W(m, name + ".weight");
    g[s].x = xs[s];
    g[s].M = segs[s].rows;
    g[s].ldx = ldx;
  }
  if (g_prof) g_prof->begin(st);
  mb_status r = check_launch(launch_qgemm_group(2, g, st), suffix);
  if (g_prof) g_prof->end(st, std::string("gemm txt+img") + suffix);
  return r;
}

// Builds the three GEMV job tables: [0] stem in_layers, [1] stem out_layers, [2] all modulations.
mb_status finalize(mb_flux* m) {
  const int64_t h = m->h();
  std::vector<GemvJob> jobs;
  std::vector<int> blocks;  // pairs (job, row0)
  auto add = [&](int table, const std::string& name, float* y, int slot) {
    const mb_weight* w = W(m, name + ".weight");
    GemvJob j = {};
    j.w = w->dev;
    j.type = w->type;
    m->gemv_kinds |= 1 << gemv_kind(w->type);
    m->gemv_smem_rb = std::max(m->gemv_smem_rb, gemv_smem_row_bytes(w->type, w->row_bytes));
    j.n_rows = (int)w->n_rows;
    j.n_cols = (int)w->n_cols;
    j.row_bytes = w->row_bytes;
    j.bias = B(m, name + ".bias");
    j.y = y;
    j.x_slot = slot;
    const int id = (int)jobs.size();
    jobs.push_back(j);
    for (int r = 0; r < j.n_rows; r += kGemvRowsPerBlock) {
      blocks.push_back(id);
      blocks.push_back(r);
    }
    m->n_jobs[table]++;
    (void)table;
  };
  const bool g = m->cfg.guidance_embed;
  m->job0[0] = 0;
  m->block0[0] = 0;
  add(0, "time_in.in_layer", m->hid, 0);
  if (g) add(0, "guidance_in.in_layer", m->hid + h, 1);
  add(0, "vector_in.in_layer", m->hid + 2 * h, 2);
  m->n_blocks[0] = (int)blocks.size() / 2;
  m->block0[1] = m->n_blocks[0];
  add(1, "time_in.out_layer", m->parts, 0);
  if (g) add(1, "guidance_in.out_layer", m->parts + h, 1);
  add(1, "vector_in.out_layer", m->parts + 2 * h, 2);
  m->n_blocks[1] = (int)blocks.size() / 2 - m->block0[1];
  m->block0[2] = m->block0[1] + m->n_blocks[1];
  m->mod_off_double.clear();
  m->mod_off_single.clear();
  int64_t off = 0;
  for (int i = 0; i < m->cfg.depth; i++) {
    m->mod_off_double.push_back(off);
    off += 12 * h;
  }
  for (int i = 0; i < m->cfg.depth_single; i++) {
    m->mod_off_single.push_back(off);
    off += 3 * h;
  }
  m->mod_off_final = off;
  off += 2 * h;
  m->mod_total = off;
  MB_TRY(dalloc(&m->mods, (size_t)off));
  for (int i = 0; i < m->cfg.depth; i++) {
    const std::string p = "double_blocks." + std::to_string(i) + ".";
    add(2, p + "img_mod.lin", m->mods + m->mod_off_double[i], 0);
    add(2, p + "txt_mod.lin", m->mods + m->mod_off_double[i] + 6 * h, 0);
  }
  for (int i = 0; i < m->cfg.depth_single; i++)
    add(2, "single_blocks." + std::to_string(i) + ".modulation.lin", m->mods + m->mod_off_single[i], 0);
  add(2, "final_layer.adaLN_modulation.1", m->mods + m->mod_off_final, 0);
  m->n_blocks[2] = (int)blocks.size() / 2 - m->block0[2];
  MB_TRY(dalloc(&m->jobs_dev, jobs.size()));
  MB_TRY(dalloc(&m->blocks_dev, blocks.size()));
  if (cudaMemcpy(m->jobs_dev, jobs.data(), jobs.size() * sizeof(GemvJob), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(m->blocks_dev, blocks.data(), blocks.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
    return set_error(MB_ERR_CUDA, "job table upload failed");
  m->finalized = true;
  return MB_OK;
}

mb_status gemv_table(const mb_flux* m, int table, const GemvInput* ins, int n_in, cudaStream_t st) {
  return check_launch(launch_gemv_batch(m->jobs_dev, m->gemv_kinds, m->blocks_dev + 2 * m->block0[table], m->n_blocks[table], ins,
                                        n_in, m->gemv_stage, m->gemv_smem_rb, st),
                      "gemv batch");
}

// The forward pass on device pointers; t / guidance are read from m->scal.
mb_status run_forward(mb_flux* m, const float* img, int64_t Li, const float* txt, int64_t Lt, const float* y,
                      cudaStream_t st) {
  const int64_t h = m->h(), H = m->H(), mh = m->mh(), L = Lt + Li, ldY = m->ldY();
  const mb_flux_config& c = m->cfg;
  // ---- conditioning vector: temb(t), temb(g), y -> stem MLPs -> all modulations
  TIMED("timestep_embedding", check_launch(launch_timestep_embedding(m->scal, 1000.f, m->temb, 256, st), "temb t"));
  if (c.guidance_embed)
    TIMED("timestep_embedding", check_launch(launch_timestep_embedding(m->scal + 1, 1000.f, m->temb + 256, 256, st), "temb g"));
  {
    GemvInput in[3] = {};
    in[0].parts[0] = m->temb;
    in[0].n_parts = 1;
    in[0].len = 256;
    in[1].parts[0] = m->temb + 256;
    in[1].n_parts = 1;
    in[1].len = 256;
    in[2].parts[0] = y;
    in[2].n_parts = 1;
    in[2].len = c.vec_in_dim;
    TIMED("gemv stems", gemv_table(m, 0, in, 3, st));
    for (int i = 0; i < 3; i++) {
      in[i].parts[0] = m->hid + i * h;
      in[i].apply_silu = 1;
      in[i].len = (int)h;
    }
    TIMED("gemv stems", gemv_table(m, 1, in, 3, st));
    GemvInput v = {};
    v.len = (int)h;
    v.parts[0] = m->parts;
    v.parts[1] = m->parts + 2 * h;
    v.n_parts = 2;
    if (c.guidance_embed) {
      v.parts[2] = m->parts + h;
      v.n_parts = 3;
    }
    v.apply_silu = 1;
    TIMED("gemv modulations", gemv_table(m, 2, &v, 1, st));
  }
  // ---- stems: txt_in, img_in into the residual stream
  TIMED("cast_f32_bf16", check_launch(launch_cast_f32_bf16(txt, Lt, c.context_in_dim, c.context_in_dim, m->txt_bf, c.context_in_dim, st),
                      "cast txt"));
  MB_TRY(linear(m, "txt_in", m->txt_bf, Lt, c.context_in_dim, m->x, h, false, MB_EPI_NONE, 0, nullptr, st));
  TIMED("cast_f32_bf16", check_launch(launch_cast_f32_bf16(img, Li, c.in_channels, c.in_channels, m->img_bf, c.in_channels, st),
                      "cast img"));
  MB_TRY(linear(m, "img_in", m->img_bf, Li, c.in_channels, m->x + Lt * h, h, false, MB_EPI_NONE, 0, nullptr, st));

  const Seg segs[2] = {{0, Lt}, {Lt, Li}};  // txt, img
  // ---- double-stream blocks: each linear of the two streams runs as one grouped launch
  for (int i = 0; i < c.depth; i++) {
    const std::string p = "double_blocks." + std::to_string(i) + ".";
    const float* md = m->mods + m->mod_off_double[i];
    const float* mos[2] = {md + 6 * h, md};  // txt_mod, img_mod
    const std::string S[2] = {"txt", "img"};
    {
      LnSegs ls = {};
      ls.n = 2;
      for (int s = 0; s < 2; s++) ls.s[s] = {segs[s].row0, segs[s].rows, mos[s], mos[s] + h};
      TIMED("ln_modulate", check_launch(launch_ln_modulate_segs(m->x, h, h, ls, m->xm, h, st), "ln_mod1"));
    }
    {
      const void* xs[2] = {m->xm, m->xm + Lt * h};
      void* ys[2] = {m->Y, m->Y + Lt * ldY};
      const float* gates[2] = {nullptr, nullptr};
      MB_TRY(linear_pair(m, p, "_attn.qkv", segs, xs, h, ys, ldY, true, MB_EPI_NONE, gates, st));
    }
    {
      QkSegs qs = {};
      qs.n = 2;
      for (int s = 0; s < 2; s++) {
        qs.s[s].row0 = segs[s].row0;
        qs.s[s].rows = segs[s].rows;
        qs.s[s].pos0 = segs[s].row0;
        qs.s[s].qs = B(m, p + S[s] + "_attn.norm.query_norm.scale");
        qs.s[s].ks = B(m, p + S[s] + "_attn.norm.key_norm.scale");
      }
      TIMED("qk_norm_rope", check_launch(launch_qk_norm_rope_segs(m->Y, ldY, (int)H, m->pe, L, qs, m->q, m->k, m->v, st),
                                         "qk_norm_rope"));
    }
    TIMED("attention", check_launch(launch_attention(m->q, m->k, m->v, (int)H, L, L, L, m->Y + 2 * h, ldY, st), "attention"));
    {
      const void* xs[2] = {m->Y + 2 * h, m->Y + Lt * ldY + 2 * h};
      void* ys[2] = {m->x, m->x + Lt * h};
      const float* gates[2] = {mos[0] + 2 * h, mos[1] + 2 * h};
      MB_TRY(linear_pair(m, p, "_attn.proj", segs, xs, ldY, ys, h, false, MB_EPI_GATE_RESIDUAL, gates, st));
    }
    {
      LnSegs ls = {};
      ls.n = 2;
      for (int s = 0; s < 2; s++) ls.s[s] = {segs[s].row0, segs[s].rows, mos[s] + 3 * h, mos[s] + 4 * h};
      TIMED("ln_modulate", check_launch(launch_ln_modulate_segs(m->x, h, h, ls, m->xm, h, st), "ln_mod2"));
    }
    {
      const void* xs[2] = {m->xm, m->xm + Lt * h};
      void* ys[2] = {m->Y + 3 * h, m->Y + Lt * ldY + 3 * h};
      const float* gates[2] = {nullptr, nullptr};
      MB_TRY(linear_pair(m, p, "_mlp.0", segs, xs, h, ys, ldY, true, MB_EPI_GELU_TANH, gates, st));
    }
    {
      const void* xs[2] = {m->Y + 3 * h, m->Y + Lt * ldY + 3 * h};
      void* ys[2] = {m->x, m->x + Lt * h};
      const float* gates[2] = {mos[0] + 5 * h, mos[1] + 5 * h};
      MB_TRY(linear_pair(m, p, "_mlp.2", segs, xs, ldY, ys, h, false, MB_EPI_GATE_RESIDUAL, gates, st));
    }
  }
  // ---- single-stream blocks over cat[txt, img] == x
  for (int i = 0; i < c.depth_single; i++) {
    const std::string p = "single_blocks." + std::to_string(i) + ".";
    const float* mo = m->mods + m->mod_off_single[i];
    TIMED("ln_modulate", check_launch(launch_ln_modulate(m->x, L, h, h, mo, mo + h, m->xm, h, st), "ln_mod"));
    MB_TRY(linear(m, p + "linear1", m->xm, L, h, m->Y, ldY, true, MB_EPI_GELU_TANH, 3 * h, nullptr, st));
    TIMED("qk_norm_rope", check_launch(launch_qk_norm_rope(m->Y, L, ldY, (int)H, B(m, p + "norm.query_norm.scale"),
                                            B(m, p + "norm.key_norm.scale"), m->pe, 0, L, m->q, m->k, m->v, st),
                        "qk_norm_rope"));
    TIMED("attention", check_launch(launch_attention(m->q, m->k, m->v, (int)H, L, L, L, m->Y + 2 * h, ldY, st), "attention"));
    MB_TRY(linear(m, p + "linear2", m->Y + 2 * h, L, ldY, m->x, h, false, MB_EPI_GATE_RESIDUAL, 0, mo + 2 * h, st));
  }
  // ---- final layer on the img rows
  {
    const float* mo = m->mods + m->mod_off_final;
    TIMED("ln_modulate", check_launch(launch_ln_modulate(m->x + Lt * h, Li, h, h, mo, mo + h, m->xm + Lt * h, h, st), "ln_final"));
    MB_TRY(linear(m, "final_layer.linear", m->xm + Lt * h, Li, h, m->pred, c.in_channels, false, MB_EPI_NONE, 0,
                  nullptr, st));
  }
  (void)mh;
  return MB_OK;
}

mb_status prepare(mb_flux* m, const float* img_ids, int64_t Li, const float* txt_ids, int64_t Lt, cudaStream_t st) {
  MB_CHECK(m->finalized || finalize(m) == MB_OK, MB_ERR_NOT_READY, mb_last_error());
  MB_CHECK(Lt >= 1 && Li >= 1 && Lt <= m->max_txt && Li <= m->max_img, MB_ERR_INVALID,
           "sequence lengths exceed the model's workspace (max_txt/max_img)");
  const int64_t L = Lt + Li;
  MB_CUDA(cudaMemcpyAsync(m->ids, txt_ids, Lt * 3 * sizeof(float), cudaMemcpyDeviceToDevice, st));
  MB_CUDA(cudaMemcpyAsync(m->ids + Lt * 3, img_ids, Li * 3 * sizeof(float), cudaMemcpyDeviceToDevice, st));
  MB_CUDA(launch_rope_table(m->ids, L, 3, m->cfg.axes_dim, m->cfg.theta, m->pe, st));
  return MB_OK;
}

}  // namespace

extern "C" {

mb_status mb_flux_create(const mb_flux_config* cfg, int64_t max_txt, int64_t max_img, mb_flux** out) {
  MB_CHECK(cfg && out, MB_ERR_INVALID, "NULL argument");
  *out = nullptr;
  MB_CHECK(cfg->num_heads > 0 && cfg->hidden_size == cfg->num_heads * 128, MB_ERR_UNSUPPORTED,
           "head_dim must be 128 (hidden_size == 128 * num_heads)");
  MB_CHECK(cfg->axes_dim[0] + cfg->axes_dim[1] + cfg->axes_dim[2] == 128, MB_ERR_INVALID, "sum(axes_dim) must be 128");
  MB_CHECK(cfg->hidden_size % 256 == 0 && cfg->mlp_hidden % 256 == 0, MB_ERR_INVALID,
           "hidden and mlp sizes must be multiples of 256");
  MB_CHECK(cfg->context_in_dim % 64 == 0 && cfg->in_channels % 64 == 0 && cfg->vec_in_dim <= 4096 &&
               cfg->vec_in_dim % 32 == 0 &&
               cfg->hidden_size <= 4096,
           MB_ERR_INVALID, "unsupported stem sizes");
  MB_CHECK(max_txt > 0 && max_img > 0, MB_ERR_INVALID, "max_txt and max_img must be positive");
  mb_flux* m = new mb_flux();
  m->cfg = *cfg;
  cudaGetDevice(&m->device);
  m->max_txt = max_txt;
  m->max_img = max_img;
  const int64_t L = max_txt + max_img, h = m->h(), H = m->H();
  mb_status s = MB_OK;
  if ((s = dalloc(&m->x, L * h)) || (s = dalloc(&m->xm, L * h)) || (s = dalloc(&m->Y, L * m->ldY())) ||
      (s = dalloc(&m->q, H * L * 128)) || (s = dalloc(&m->k, H * L * 128)) || (s = dalloc(&m->v, H * L * 128)) ||
      (s = dalloc(&m->pe, L * 256)) || (s = dalloc(&m->ids, L * 3)) ||
      (s = dalloc(&m->txt_bf, max_txt * cfg->context_in_dim)) || (s = dalloc(&m->img_bf, max_img * cfg->in_channels)) ||
      (s = dalloc(&m->pred, max_img * cfg->in_channels)) || (s = dalloc(&m->scal, 8)) ||
      (s = dalloc(&m->counter, 1)) || (s = dalloc(&m->temb, 512)) || (s = dalloc(&m->hid, 3 * h)) ||
      (s = dalloc(&m->parts, 3 * h)) || (s = dalloc(&m->gemv_stage, gemv_stage_floats()))) {
    mb_flux_destroy(m);
    return s;
  }
  cudaMemset(m->hid, 0, 3 * h * sizeof(float));
  cudaMemset(m->parts, 0, 3 * h * sizeof(float));
  *out = m;
  return MB_OK;
}

mb_status mb_flux_destroy(mb_flux* m) {
  if (!m) return MB_OK;
  if (m->graph) cudaGraphExecDestroy(m->graph);
  for (auto& kv : m->mats) mb_weight_destroy(kv.second);
  for (auto& kv : m->vecs) cudaFree(kv.second.dev);
  void* bufs[] = {m->x, m->xm, m->Y, m->q, m->k, m->v, m->pe, m->ids, m->txt_bf, m->img_bf, m->pred, m->scal,
                  m->counter, m->sched, m->temb, m->hid, m->parts, m->mods, m->jobs_dev, m->blocks_dev,
                  m->gemv_stage};
  for (void* b : bufs)
    if (b) cudaFree(b);
  delete m;
  return MB_OK;
}

mb_status mb_flux_set_tensor(mb_flux* m, const char* name, int ggml_type, int64_t n_rows, int64_t n_cols,
                             const void* data, size_t nbytes, int data_on_device) {
  MB_CHECK(m && name && data, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(!m->finalized, MB_ERR_INVALID, "tensors cannot be replaced after the first forward");
  const std::string n(name);
  const auto exp = expected_tensors(m->cfg);
  const std::vector<int64_t>* shape = nullptr;
  for (const auto& e : exp)
    if (e.first == n) shape = &e.second;
  MB_CHECK(shape, MB_ERR_INVALID, "unknown FLUX tensor name '" + n + "'");
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
  const bool gemv_only = n.find("_mod.lin") != std::string::npos || n.find("modulation") != std::string::npos ||
                         n.rfind("time_in", 0) == 0 || n.rfind("vector_in", 0) == 0 || n.rfind("guidance_in", 0) == 0;
  mb_weight* w = nullptr;
  MB_TRY(upload_matrix(ggml_type, n_rows, n_cols, data, nbytes, data_on_device, !gemv_only, &w));
  auto it = m->mats.find(n);
  if (it != m->mats.end()) mb_weight_destroy(it->second);
  m->mats[n] = w;
  return MB_OK;
}

mb_status mb_flux_lora_merge(mb_flux* m, const char* name, int64_t row_offset, int64_t rows, const float* A,
                             const float* B, int rank, float scale, void* stream) {
  MB_CHECK(m && name, MB_ERR_INVALID, "NULL argument");
  auto it = m->mats.find(name);
  MB_CHECK(it != m->mats.end(), MB_ERR_INVALID, std::string("no FLUX weight matrix '") + name + "' is loaded");
  return mb_weight_lora_merge(it->second, row_offset, rows, A, B, rank, scale, stream);
}

mb_status mb_flux_missing(const mb_flux* m, char* buf, size_t buflen) {
  MB_CHECK(m && buf && buflen > 0, MB_ERR_INVALID, "NULL argument");
  std::string s;
  for (const auto& e : expected_tensors(m->cfg)) {
    const bool have = e.second.size() == 1 ? m->vecs.count(e.first) > 0 : m->mats.count(e.first) > 0;
    if (!have) s += e.first + "\n";
  }
  const size_t n = s.size() < buflen - 1 ? s.size() : buflen - 1;
  memcpy(buf, s.data(), n);
  buf[n] = 0;
  return MB_OK;
}

static mb_status check_complete(const mb_flux* m) {
  char buf[256];
  mb_flux_missing(m, buf, sizeof(buf));
  MB_CHECK(buf[0] == 0, MB_ERR_NOT_READY, std::string("FLUX model is missing tensors, first: ") + buf);
  return MB_OK;
}

mb_status mb_flux_forward(mb_flux* m, const float* img, const float* img_ids, int64_t L_img, const float* txt,
                          const float* txt_ids, int64_t L_txt, float t, const float* y, float guidance, float* pred,
                          void* stream) {
  MB_CHECK(m && img && img_ids && txt && txt_ids && y && pred, MB_ERR_INVALID, "NULL argument");
  MB_TRY(check_complete(m));
  cudaStream_t st = (cudaStream_t)stream;
  MB_TRY(prepare(m, img_ids, L_img, txt_ids, L_txt, st));
  MB_CUDA(launch_set_scalars(m->scal, t, guidance, st));
  OpProfiler prof;
  if (profile_requested()) g_prof = &prof;
  mb_status fs = run_forward(m, img, L_img, txt, L_txt, y, st);
  if (g_prof) {
    g_prof = nullptr;
    prof.report();
  }
  MB_TRY(fs);
  MB_CUDA(cudaMemcpyAsync(pred, m->pred, L_img * m->cfg.in_channels * sizeof(float), cudaMemcpyDeviceToDevice, st));
  return MB_OK;
}

mb_status mb_flux_denoise_ex(mb_flux* m, float* img, const float* img_ids, int64_t L_img, const float* txt,
                             const float* txt_ids, int64_t L_txt, const float* y, const double* timesteps,
                             int n_timesteps, float guidance, const mb_inpaint* inpaint, mb_step_callback on_step,
                             void* user, void* stream) {
  MB_CHECK(m && img && img_ids && txt && txt_ids && y && timesteps, MB_ERR_INVALID, "NULL argument");
  MB_CHECK(n_timesteps >= 2, MB_ERR_INVALID, "need at least two timesteps");
  MB_CHECK(!inpaint || (inpaint->mask && inpaint->original && inpaint->noise), MB_ERR_INVALID,
           "inpaint needs mask, original and noise");
  MB_TRY(check_complete(m));
  cudaStream_t st = (cudaStream_t)stream;
  MB_TRY(prepare(m, img_ids, L_img, txt_ids, L_txt, st));
  if (m->sched_cap < n_timesteps) {
    if (m->sched) cudaFree(m->sched);
    m->sched = nullptr;
    const int cap = n_timesteps > 1024 ? n_timesteps : 1024;  // keeps the pointer (and the graph) stable
    MB_TRY(dalloc(&m->sched, (size_t)cap));
    m->sched_cap = cap;
  }
  MB_CUDA(cudaMemcpyAsync(m->sched, timesteps, n_timesteps * sizeof(double), cudaMemcpyHostToDevice, st));
  MB_CUDA(cudaMemsetAsync(m->counter, 0, sizeof(int), st));
  MB_CUDA(launch_set_scalars(m->scal, (float)timesteps[0], guidance, st));
  const int64_t n_img = L_img * m->cfg.in_channels;
  const void* key[7] = {img, txt, y, m->sched, inpaint ? inpaint->mask : nullptr,
                        inpaint ? inpaint->original : nullptr, inpaint ? inpaint->noise : nullptr};
  const bool reuse = m->graph && m->graph_lt == L_txt && m->graph_li == L_img &&
                     memcmp(key, m->graph_key, sizeof(key)) == 0;
  if (!reuse) {
    if (m->graph) {
      cudaGraphExecDestroy(m->graph);
      m->graph = nullptr;
    }
    // Eager warm-up of the step so every kernel attribute is set before capture.
    MB_CUDA(launch_step_prologue(m->sched, m->counter, m->scal, st));
    MB_TRY(run_forward(m, img, L_img, txt, L_txt, y, st));
    MB_CUDA(cudaMemsetAsync(m->counter, 0, sizeof(int), st));
    MB_CUDA(cudaStreamSynchronize(st));
    cudaStream_t cs;
    MB_CUDA(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    cudaGraph_t g;
    MB_CUDA(cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal));
    launch_step_prologue(m->sched, m->counter, m->scal, cs);
    mb_status s = run_forward(m, img, L_img, txt, L_txt, y, cs);
    cudaError_t le = launch_euler_dev(img, m->pred, n_img, m->scal + 2, cs);
    if (le == cudaSuccess && inpaint)
      le = launch_inpaint_blend(img, n_img, m->scal, inpaint->mask, inpaint->original, inpaint->noise, cs);
    cudaError_t ce = cudaStreamEndCapture(cs, &g);
    cudaStreamDestroy(cs);
    if (s != MB_OK) return s;
    MB_CUDA(le);
    MB_CUDA(ce);
    cudaError_t ie = cudaGraphInstantiate(&m->graph, g, 0);
    cudaGraphDestroy(g);
    MB_CUDA(ie);
    m->graph_lt = L_txt;
    m->graph_li = L_img;
    memcpy(m->graph_key, key, sizeof(key));
  }
  MB_CUDA(enqueue_steps(m->graph, n_timesteps - 1, on_step, user, st));
  return MB_OK;
}

mb_status mb_flux_denoise(mb_flux* m, float* img, const float* img_ids, int64_t L_img, const float* txt,
                          const float* txt_ids, int64_t L_txt, const float* y, const double* timesteps,
                          int n_timesteps, float guidance, void* stream) {
  return mb_flux_denoise_ex(m, img, img_ids, L_img, txt, txt_ids, L_txt, y, timesteps, n_timesteps, guidance,
                            nullptr, nullptr, nullptr, stream);
}

}  // extern "C"
