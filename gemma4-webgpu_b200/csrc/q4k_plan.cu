// Plans: a recorded sequence of matmul-path operations replayed with a fixed
// number of launches (2 per stage), the way src/engine.ts records a token's
// passes into one command encoder with pre-built bind groups
// (encodeTransformerPass, :1466-1626) and submits it once (:1748).
//
// A plan has stages.  Inside a stage every operation is independent: one
// activation-preparation launch prepares every distinct GEMV input (and
// evaluates gelu_mul ops whose output feeds a GEMV of the same stage), then
// one engine launch runs every GEMV and the LM-head selection of the stage
// over one shared work list.  Stage s+1 starts after stage s has finished.
// A stage that mixes weight formats (Q4_K and Q6_K matrices) runs as one
// engine launch per format, back to back.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <vector>

#include "q4k_ctx.cuh"

using namespace q4k;

namespace {

struct PlanGemv {
  const uint8_t* w;
  const float* x;
  float* y;
  uint32_t M, N;
  uint32_t fmt;  // WeightFormat of w
};

struct PlanGelu {
  const float* gate;
  const float* up;
  float* act;
  uint32_t n;
};

struct PlanSelect {
  const uint8_t* w;
  const float* x;
  uint32_t V, N;
  float cap;
  uint32_t row_offset;
  float* logits;
  float* cand_val;
  uint32_t* cand_idx;
  uint32_t* argmax;
  uint32_t fmt;
};

struct Stage {
  std::vector<PlanGemv> gemvs;
  std::vector<PlanGelu> gelus;
  std::vector<PlanSelect> selects;
  // filled by commit
  EngineTask* tasks_dev = nullptr;
  CUtensorMap* maps_dev = nullptr;
  XJob* jobs_dev = nullptr;
  CtaSched* sched_dev = nullptr;
  uint32_t n_tasks = 0, n_jobs = 0, total_items = 0, total_cost = 0, grid = 0, select_task = 0;
  bool prep = false;  // activations prepared inside the engine launch (no preparation launch)
  uint32_t ksplit = 0;  // warps sharing each tile (long rows only; see TaskList::ksplit)
  uint32_t fmt = kFmtQ4K;  // after commit: the weight format of every task of this launch unit
  bool pairs = false;      // after commit: every task fills both super-blocks of its stages (TaskList::pairs)
  // GEMM plans (batch >= kGemmMinRows): one preparation launch over the
  // stage's activation jobs, one multi-matrix GEMM launch over its tiles
  GemmJob* gjobs_dev = nullptr;
  GemmTask* gtasks_dev = nullptr;
  uint2* tiles_dev = nullptr;
  uint32_t n_gjobs = 0, n_tiles = 0;
  uint32_t gjob_max_n = 0;      // widest activation job of the stage
  uint32_t gsplit = 1;          // K split of every matrix of the stage (1 or 2)
  uint32_t n_gkeys = 0;         // activation jobs; the K-split zeroing jobs follow them
  bool gjobs_aligned = false;   // every job pointer 16-byte aligned (single-read preparation)
};

// Commit splits each recorded stage into launch units of one weight format
// (Q4_K first); a gelu_mul goes with every unit that reads its output (the
// Q4_K unit if none does).
std::vector<Stage> split_by_format(const std::vector<Stage>& stages) {
  std::vector<Stage> units;
  for (const Stage& st : stages) {
    Stage u[2];
    u[1].fmt = kFmtQ6K;
    for (const PlanGemv& g : st.gemvs) u[g.fmt == kFmtQ6K].gemvs.push_back(g);
    for (const PlanSelect& q : st.selects) u[q.fmt == kFmtQ6K].selects.push_back(q);
    for (const PlanGelu& gl : st.gelus) {
      bool used[2] = {false, false};
      for (int f = 0; f < 2; ++f) {
        for (const PlanGemv& g : u[f].gemvs) used[f] |= (g.x == gl.act);
        for (const PlanSelect& q : u[f].selects) used[f] |= (q.x == gl.act);
      }
      if (!used[0] && !used[1]) used[0] = true;
      for (int f = 0; f < 2; ++f)
        if (used[f]) u[f].gelus.push_back(gl);
    }
    for (int f = 0; f < 2; ++f)
      if (!u[f].gemvs.empty() || !u[f].selects.empty() || !u[f].gelus.empty()) units.push_back(u[f]);
  }
  return units;
}

}  // namespace

struct q4k_plan {
  q4k_ctx* ctx = nullptr;
  uint32_t batch = 1;
  bool gemm = false;   // batch >= kGemmMinRows: stages run on the tcgen05 GEMM
  uint32_t parts = 1;  // GEMM plans: operand rows per activation row (1: f16, 2: exact f16 hi + lo)
  std::vector<Stage> stages;
  bool committed = false;
  void* mem = nullptr;  // one allocation: descriptors + prepared activations
  size_t bytes = 0;
};

namespace {

Stage* stage_of(q4k_plan* p, uint32_t s) {
  if (s >= 64) return nullptr;
  if (p->stages.size() <= s) p->stages.resize(s + 1);
  return &p->stages[s];
}

int check_plan(q4k_plan* p) {
  if (!p) return Q4K_ERR_INVALID_ARG;
  if (p->committed) return ctx_fail(p->ctx, Q4K_ERR_INVALID_ARG, "plan already committed");
  return Q4K_OK;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Largest batch of a GEMM plan (16-bit token-tile indices in the tile table).
constexpr uint32_t kPlanMaxGemmRows = 8192;

// Plan tasks carry their own maps; the launch parameter is unused.
const CUtensorMap kNoMap{};

}  // namespace

extern "C" {

int q4k_plan_create(q4k_ctx* ctx, uint32_t batch, q4k_plan** out) {
  if (!ctx || !out) return Q4K_ERR_INVALID_ARG;
  *out = nullptr;
  if (batch == 0 || (batch > (uint32_t)kMaxTokens && batch < kGemmMinRows) || batch > kPlanMaxGemmRows)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "plan batch=%u outside [1, %d] and [%u, %u]", batch, kMaxTokens,
                    kGemmMinRows, kPlanMaxGemmRows);
  q4k_plan* p = new q4k_plan();
  p->ctx = ctx;
  p->batch = batch;
  p->gemm = batch >= kGemmMinRows;
  *out = p;
  return Q4K_OK;
}

int q4k_plan_gemm_exact(q4k_plan* p, int exact) {
  int rc = check_plan(p);
  if (rc != Q4K_OK) return rc;
  if (!p->gemm) return ctx_fail(p->ctx, Q4K_ERR_INVALID_ARG, "batch-%u plans run on the GEMV engine", p->batch);
  p->parts = exact ? 2u : 1u;
  return Q4K_OK;
}

void q4k_plan_destroy(q4k_plan* p) {
  if (!p) return;
  if (p->mem) cudaFree(p->mem);
  delete p;
}

static int plan_gemv(q4k_plan* p, uint32_t stage, const void* w, const float* x, float* y, uint32_t M, uint32_t N,
              uint32_t fmt) {
  int rc = check_plan(p);
  if (rc != Q4K_OK) return rc;
  q4k_ctx* ctx = p->ctx;
  if (!w || !x || !y) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (M == 0 || N == 0 || N % Q4K_QK != 0)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "bad shape M=%u N=%u (N must be a multiple of 256)", M, N);
  if (!aligned16(w) || !aligned16(x) || !aligned16(y))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "pointers must be 16-byte aligned");
  if (p->gemm && fmt != kFmtQ4K)
    return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "batch-%u plans take Q4_K matrices only", p->batch);
  Stage* st = stage_of(p, stage);
  if (!st) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "stage %u out of range", stage);
  st->gemvs.push_back({static_cast<const uint8_t*>(w), x, y, M, N, fmt});
  return Q4K_OK;
}

int q4k_plan_gemv(q4k_plan* p, uint32_t stage, const void* w, const float* x, float* y, uint32_t M, uint32_t N) {
  return plan_gemv(p, stage, w, x, y, M, N, kFmtQ4K);
}

int q4k_plan_gemv_q6k(q4k_plan* p, uint32_t stage, const void* w_dev, const float* x, float* y, uint32_t M,
                      uint32_t N) {
  return plan_gemv(p, stage, w_dev, x, y, M, N, kFmtQ6K);
}

int q4k_plan_gelu_mul(q4k_plan* p, uint32_t stage, const float* gate, const float* up, float* act, uint32_t n) {
  int rc = check_plan(p);
  if (rc != Q4K_OK) return rc;
  q4k_ctx* ctx = p->ctx;
  if (!gate || !up || !act) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (n == 0 || n % Q4K_QK != 0)
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "plan gelu_mul size %u must be a multiple of 256", n);
  if (!aligned16(gate) || !aligned16(up) || !aligned16(act))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "gelu_mul pointers must be 16-byte aligned");
  Stage* st = stage_of(p, stage);
  if (!st) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "stage %u out of range", stage);
  st->gelus.push_back({gate, up, act, n});
  return Q4K_OK;
}

static int plan_lmhead(q4k_plan* p, uint32_t stage, const void* w, const float* x, uint32_t V, uint32_t N, float cap,
                uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx, uint32_t* argmax,
                uint32_t fmt) {
  int rc = check_plan(p);
  if (rc != Q4K_OK) return rc;
  q4k_ctx* ctx = p->ctx;
  if (p->batch != 1) return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "the fused LM head takes batch 1");
  if (!w || !x || !cand_val || !cand_idx || !argmax) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "null pointer");
  if (V == 0 || N == 0 || N % Q4K_QK != 0) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "bad shape V=%u N=%u", V, N);
  if ((uint64_t)row_offset + V >= (1ull << 31))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "row_offset + V must be < 2^31");
  if (!aligned16(w) || !aligned16(x) || (logits && !aligned16(logits)))
    return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "pointers must be 16-byte aligned");
  Stage* st = stage_of(p, stage);
  if (!st) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "stage %u out of range", stage);
  if (!st->selects.empty()) return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "one LM head per plan stage");
  st->selects.push_back({static_cast<const uint8_t*>(w), x, V, N, cap, row_offset, logits, cand_val, cand_idx,
                         argmax, fmt});
  return Q4K_OK;
}

int q4k_plan_lmhead(q4k_plan* p, uint32_t stage, const void* w, const float* x, uint32_t V, uint32_t N, float cap,
                    uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx, uint32_t* argmax) {
  return plan_lmhead(p, stage, w, x, V, N, cap, row_offset, logits, cand_val, cand_idx, argmax, kFmtQ4K);
}

int q4k_plan_lmhead_q6k(q4k_plan* p, uint32_t stage, const void* w_dev, const float* x, uint32_t V, uint32_t N,
                        float cap, uint32_t row_offset, float* logits, float* cand_val, uint32_t* cand_idx,
                        uint32_t* argmax) {
  return plan_lmhead(p, stage, w_dev, x, V, N, cap, row_offset, logits, cand_val, cand_idx, argmax, kFmtQ6K);
}

static int commit_gemm(q4k_plan* p);

int q4k_plan_commit(q4k_plan* p) {
  int rc = check_plan(p);
  if (rc != Q4K_OK) return rc;
  if (p->gemm) return commit_gemm(p);
  q4k_ctx* ctx = p->ctx;
  const uint32_t B = p->batch;
  p->stages = split_by_format(p->stages);
  // Per stage: one preparation job per distinct (input, N); a gelu_mul's
  // output is a GEMV input of its stage.
  struct JobKey {
    const float* x;
    uint32_t N;
    int gelu;  // index into gelus, or -1
  };
  std::vector<std::vector<JobKey>> keys(p->stages.size());
  std::vector<std::vector<EngineTask>> tasks(p->stages.size());
  size_t xbytes = 0, desc_bytes = 0;
  for (size_t s = 0; s < p->stages.size(); ++s) {
    Stage& st = p->stages[s];
    auto job_for = [&](const float* x, uint32_t N) -> int {
      for (size_t j = 0; j < keys[s].size(); ++j)
        if (keys[s][j].x == x && keys[s][j].N == N) return (int)j;
      int gelu = -1;
      for (size_t g = 0; g < st.gelus.size(); ++g)
        if (st.gelus[g].act == x) {
          if (st.gelus[g].n != N) return -2;
          gelu = (int)g;
        }
      keys[s].push_back({x, N, gelu});
      return (int)keys[s].size() - 1;
    };
    uint32_t items = 0, cost = 0;
    for (const PlanGemv& g : st.gemvs) {
      const int j = job_for(g.x, g.N);
      if (j < 0) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "gelu_mul output size differs from a GEMV's N");
      EngineTask t{};
      t.w = g.w;
      t.y = g.y;
      t.M = g.M;
      t.N = g.N;
      t.kind = kTaskPlain;
      t.item_begin = items;
      t.cost_begin = cost;
      items += tiles_of(g.M);
      cost += tiles_of(g.M) * item_cost(g.N, kTaskPlain);
      t.item_end = items;
      t.aux = (uint32_t)j;  // job index until the buffers are laid out
      tasks[s].push_back(t);
    }
    for (const PlanSelect& q : st.selects) {
      st.select_task = (uint32_t)tasks[s].size();
      const int j = job_for(q.x, q.N);
      if (j < 0) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "gelu_mul output size differs from the LM head's N");
      EngineTask t{};
      t.w = q.w;
      t.logits = q.logits;
      t.cand_val = q.cand_val;
      t.cand_idx = q.cand_idx;
      t.argmax = q.argmax;
      t.M = q.V;
      t.N = q.N;
      t.kind = kTaskSelect;
      t.row_offset = q.row_offset;
      t.cap = q.cap;
      t.item_begin = items;
      t.cost_begin = cost;
      items += tiles_of(q.V);
      cost += tiles_of(q.V) * item_cost(q.N, kTaskSelect);
      t.item_end = items;
      t.aux = (uint32_t)j;
      tasks[s].push_back(t);
    }
    // gelu_mul ops nobody consumes still run (their act output is written)
    for (size_t g = 0; g < st.gelus.size(); ++g) {
      bool used = false;
      for (const JobKey& k : keys[s]) used |= (k.gelu == (int)g);
      if (!used) keys[s].push_back({st.gelus[g].act, st.gelus[g].n, (int)g});
    }
    st.total_items = items;
    st.total_cost = cost;
    // Rows of >= 16 super-blocks (the FFN down projection) make few, long
    // items: a stage of only such GEMVs shares each tile across 4 warps,
    // each taking a quarter of the row, so the items balance over the warps.
    {
      bool long_rows = B <= 4 && st.selects.empty() && !tasks[s].empty() && st.fmt == kFmtQ4K;
      for (const EngineTask& t : tasks[s]) {
        const uint32_t nb = t.N / Q4K_QK;
        long_rows = long_rows && nb >= 16 && nb % 4 == 0;
      }
      st.ksplit = long_rows ? 4u : 0u;
    }
    st.n_tasks = (uint32_t)tasks[s].size();
    st.n_jobs = (uint32_t)keys[s].size();
    st.grid = items ? engine_grid(items, ctx->sm_count) : 0;
    for (const JobKey& k : keys[s]) xbytes += align_up(xfrag_bytes(k.N, B), 256) + 256;
    desc_bytes += align_up(sizeof(EngineTask) * st.n_tasks, 256) + align_up(sizeof(CUtensorMap) * 2 * st.n_tasks, 256) +
                  align_up(sizeof(XJob) * st.n_jobs, 256) + align_up(sizeof(CtaSched) * st.grid, 256);
  }
  p->bytes = desc_bytes + xbytes;
  if (p->bytes == 0) {
    p->committed = true;
    return Q4K_OK;
  }
  cudaError_t e = cudaMalloc(&p->mem, p->bytes);
  if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit allocation");
  char* cur = static_cast<char*>(p->mem);
  char* xcur = cur + desc_bytes;
  for (size_t s = 0; s < p->stages.size(); ++s) {
    Stage& st = p->stages[s];
    std::vector<XJob> jobs(st.n_jobs);
    for (uint32_t j = 0; j < st.n_jobs; ++j) {
      const JobKey& k = keys[s][j];
      XJob& J = jobs[j];
      J = XJob{};
      J.N = k.N;
      if (k.gelu >= 0) {
        const PlanGelu& g = st.gelus[k.gelu];
        J.mode = 1;
        J.gate = g.gate;
        J.up = g.up;
        J.act = g.act;
      } else {
        J.mode = 0;
        J.x = k.x;
      }
      J.xfrag = reinterpret_cast<uint2*>(xcur);
      xcur += align_up(xfrag_bytes(k.N, B), 256);
      J.inv_scale = reinterpret_cast<float*>(xcur);
      xcur += 256;
    }
    for (EngineTask& t : tasks[s]) {
      const XJob& J = jobs[t.aux];
      t.xfrag = J.xfrag;
      t.inv_scale = J.inv_scale;  // t.aux keeps the job index (the CTA schedules name jobs by it)
    }
    // the weight tensor maps of each task (Q6_K: body map, then d-plane map), in the plan's memory
    const uint32_t mpt = st.fmt == kFmtQ6K ? 2u : 1u;
    st.maps_dev = reinterpret_cast<CUtensorMap*>(cur);
    cur += align_up(sizeof(CUtensorMap) * 2 * st.n_tasks, 256);
    std::vector<CUtensorMap> maps(mpt * st.n_tasks);
    for (uint32_t i = 0; i < st.n_tasks; ++i) {
      EngineTask& t = tasks[s][i];
      e = st.fmt == kFmtQ6K ? encode_q6k_maps(&maps[mpt * i], t.w, t.M, t.N, &t.tile_bytes)
                            : encode_weight_map(&maps[i], t.w, t.M, t.N, &t.tile_bytes);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit weight tensor map");
      t.tmap = st.maps_dev + mpt * i;
    }
    st.pairs = st.fmt == kFmtQ4K && st.n_tasks > 0;
    for (const EngineTask& t : tasks[s]) st.pairs = st.pairs && pairs_of(t.N, st.ksplit, t.tile_bytes);
    if (st.n_tasks) {
      e = cudaMemcpy(st.maps_dev, maps.data(), sizeof(CUtensorMap) * maps.size(), cudaMemcpyHostToDevice);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit upload");
    }
    st.tasks_dev = reinterpret_cast<EngineTask*>(cur);
    cur += align_up(sizeof(EngineTask) * st.n_tasks, 256);
    st.jobs_dev = reinterpret_cast<XJob*>(cur);
    cur += align_up(sizeof(XJob) * st.n_jobs, 256);
    st.sched_dev = reinterpret_cast<CtaSched*>(cur);
    cur += align_up(sizeof(CtaSched) * st.grid, 256);
    if (st.grid) {
      std::vector<CtaSched> sched(st.grid);
      engine_schedule(tasks[s].data(), st.n_tasks, st.total_cost, st.total_items, B, st.grid,
                      engine_xcache_bytes(!st.selects.empty(), st.fmt), sched.data());
      // Prepare activations inside the engine when every CTA caches every
      // activation it uses and each stored gelu_mul output has a CTA that
      // prepares it (the first such CTA stores it).
      st.prep = schedule_covers_tasks(tasks[s].data(), st.n_tasks, sched.data(), st.grid);
      for (uint32_t j = 0; st.prep && j < st.n_jobs; ++j) {
        if (!(jobs[j].mode && jobs[j].act)) continue;
        bool owned = false;
        for (uint32_t b = 0; b < st.grid && !owned; ++b)
          for (uint32_t k = 0; k < sched[b].nx; ++k)
            if (sched[b].xjob[k] == j) {
              sched[b].act_mask |= 1u << k;
              owned = true;
              break;
            }
        if (!owned) st.prep = false;
      }
      e = cudaMemcpy(st.sched_dev, sched.data(), sizeof(CtaSched) * st.grid, cudaMemcpyHostToDevice);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit upload");
    }
    if (st.n_tasks) {
      e = cudaMemcpy(st.tasks_dev, tasks[s].data(), sizeof(EngineTask) * st.n_tasks, cudaMemcpyHostToDevice);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit upload");
    }
    if (st.n_jobs) {
      e = cudaMemcpy(st.jobs_dev, jobs.data(), sizeof(XJob) * st.n_jobs, cudaMemcpyHostToDevice);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit upload");
    }
  }
  p->committed = true;
  ctx->err[0] = 0;
  return Q4K_OK;
}

// GEMM plans: per stage, one job per distinct activation (x, or a gelu_mul
// output that a GEMM of the stage reads), its B operand in the plan's
// memory, one task per matrix, and the tile table of the stage's single
// GEMM launch: every (weight-row tile, token tile) of every matrix, longest
// rows first so the last wave holds the short tiles.
static int commit_gemm(q4k_plan* p) {
  q4k_ctx* ctx = p->ctx;
  const uint32_t T = p->batch, parts = p->parts, tt = gemm_tile_tokens(parts, T), tr = gemm_tile_rows();
  struct Key {
    const float* x;
    uint32_t N;
    int gelu;
  };
  std::vector<std::vector<Key>> keys(p->stages.size());
  std::vector<std::vector<uint32_t>> task_job(p->stages.size());
  size_t desc = 0, ops = 0;
  for (size_t s = 0; s < p->stages.size(); ++s) {
    Stage& st = p->stages[s];
    if (!st.selects.empty()) return ctx_fail(ctx, Q4K_ERR_UNSUPPORTED, "GEMM plans have no fused LM head");
    auto job_for = [&](const float* x, uint32_t N) -> int {
      for (size_t j = 0; j < keys[s].size(); ++j)
        if (keys[s][j].x == x && keys[s][j].N == N) return (int)j;
      int gelu = -1;
      for (size_t g = 0; g < st.gelus.size(); ++g)
        if (st.gelus[g].act == x) {
          if (st.gelus[g].n != N) return -2;
          gelu = (int)g;
        }
      keys[s].push_back({x, N, gelu});
      return (int)keys[s].size() - 1;
    };
    for (const PlanGemv& g : st.gemvs) {
      const int j = job_for(g.x, g.N);
      if (j < 0) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "gelu_mul output size differs from a GEMV's N");
      task_job[s].push_back((uint32_t)j);
      st.n_tiles += ((g.M + tr - 1) / tr) * ((T + tt - 1) / tt);
    }
    for (size_t g = 0; g < st.gelus.size(); ++g) {
      bool used = false;
      for (const Key& k : keys[s]) used |= (k.gelu == (int)g);
      if (!used) keys[s].push_back({st.gelus[g].act, st.gelus[g].n, (int)g});
    }
    // A stage of long-K matrices that fills less than whole rounds of the
    // SMs (the downs at small T: 210 tiles of 96 K steps on 148 SMs) runs
    // each matrix as two K halves accumulating into its zeroed output.  The
    // output is then 0 + a + b in either order, which fp32 gives exactly.
    {
      bool can = !st.gemvs.empty();
      uint32_t steps = 0;
      for (const PlanGemv& g : st.gemvs) {
        can = can && g.N % 512 == 0 && g.N >= 2048;
        steps = steps > g.N / 64 ? steps : g.N / 64;
      }
      const uint32_t sms = (uint32_t)(ctx->sm_count > 0 ? ctx->sm_count : 1);
      auto rounds = [&](uint32_t n) { return (n + sms - 1) / sms; };
      st.gsplit = can && rounds(2 * st.n_tiles) * (steps / 2) < rounds(st.n_tiles) * steps ? 2 : 1;
    }
    st.n_tiles *= st.gsplit;
    st.n_tasks = (uint32_t)st.gemvs.size() * st.gsplit;
    st.n_gkeys = (uint32_t)keys[s].size();
    st.n_gjobs = st.n_gkeys + (st.gsplit > 1 ? (uint32_t)st.gemvs.size() : 0u);
    desc += align_up(sizeof(GemmTask) * st.n_tasks, 256) + align_up(sizeof(GemmJob) * st.n_gjobs, 256) +
            align_up(sizeof(CUtensorMap) * (st.n_tasks + st.n_gjobs), 256) + align_up(sizeof(uint2) * st.n_tiles, 256);
    for (const Key& k : keys[s]) ops += align_up(gemm_operand_bytes(k.N, T, parts), 256) + align_up(4ull * T, 256);
  }
  p->bytes = desc + ops;
  if (p->bytes == 0) {
    p->committed = true;
    return Q4K_OK;
  }
  cudaError_t e = cudaMalloc(&p->mem, p->bytes);
  if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit allocation");
  char* cur = static_cast<char*>(p->mem);
  char* ocur = cur + desc;
  for (size_t s = 0; s < p->stages.size(); ++s) {
    Stage& st = p->stages[s];
    CUtensorMap* maps_dev = reinterpret_cast<CUtensorMap*>(cur);
    cur += align_up(sizeof(CUtensorMap) * (st.n_tasks + st.n_gjobs), 256);
    st.gtasks_dev = reinterpret_cast<GemmTask*>(cur);
    cur += align_up(sizeof(GemmTask) * st.n_tasks, 256);
    st.gjobs_dev = reinterpret_cast<GemmJob*>(cur);
    cur += align_up(sizeof(GemmJob) * st.n_gjobs, 256);
    st.tiles_dev = reinterpret_cast<uint2*>(cur);
    cur += align_up(sizeof(uint2) * st.n_tiles, 256);
    std::vector<CUtensorMap> maps(st.n_tasks + st.n_gjobs);
    std::vector<GemmJob> jobs(st.n_gjobs);
    for (uint32_t j = 0; j < st.n_gkeys; ++j) {
      const Key& k = keys[s][j];
      GemmJob& J = jobs[j];
      J = GemmJob{};
      J.N = k.N;
      if (k.gelu >= 0) {
        const PlanGelu& g = st.gelus[k.gelu];
        J.mode = 1;
        J.gate = g.gate;
        J.up = g.up;
        J.act = g.act;
      } else {
        J.x = k.x;
      }
      J.operand = ocur;
      ocur += align_up(gemm_operand_bytes(k.N, T, parts), 256);
      J.inv_scale = reinterpret_cast<float*>(ocur);
      ocur += align_up(4ull * T, 256);
      e = gemm_operand_map(&maps[st.n_tasks + j], J.operand, k.N, T, parts);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit activation tensor map");
      st.gjob_max_n = st.gjob_max_n > k.N ? st.gjob_max_n : k.N;
      const uintptr_t bits = reinterpret_cast<uintptr_t>(J.x) | reinterpret_cast<uintptr_t>(J.gate) |
                             reinterpret_cast<uintptr_t>(J.up) | reinterpret_cast<uintptr_t>(J.act) |
                             reinterpret_cast<uintptr_t>(J.operand);
      if (j == 0) st.gjobs_aligned = true;
      st.gjobs_aligned = st.gjobs_aligned && (bits & 15u) == 0;
    }
    // the K-split zeroing jobs: one per matrix output
    for (uint32_t i = 0; st.gsplit > 1 && i < st.gemvs.size(); ++i) {
      GemmJob& J = jobs[st.n_gkeys + i];
      J = GemmJob{};
      J.mode = 2;
      J.act = st.gemvs[i].y;
      J.N = st.gemvs[i].M;
    }
    std::vector<GemmTask> tasks(st.n_tasks);
    std::vector<uint2> tiles;
    tiles.reserve(st.n_tiles);
    for (uint32_t i = 0; i < st.n_tasks; ++i) {
      const PlanGemv& g = st.gemvs[i / st.gsplit];
      const uint32_t j = task_job[s][i / st.gsplit], h = i % st.gsplit;
      e = gemm_weight_map(&maps[i], g.w, g.M, g.N);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit weight tensor map");
      GemmTask& t = tasks[i];
      t = GemmTask{};
      t.amap = maps_dev + i;
      t.bmap = maps_dev + st.n_tasks + j;
      t.y = g.y;
      t.inv_scale = jobs[j].inv_scale;
      t.M = g.M;
      t.N = g.N / st.gsplit;
      t.k0 = h * t.N;
      t.accumulate = st.gsplit > 1;
      t.T = T;
      t.tile_tokens = tt;
      for (uint32_t r = 0; r < (g.M + tr - 1) / tr; ++r)
        for (uint32_t q = 0; q < (T + tt - 1) / tt; ++q) tiles.push_back(make_uint2(i, r | (q << 16)));
    }
    std::stable_sort(tiles.begin(), tiles.end(),
                     [&](const uint2& a, const uint2& b) { return tasks[a.x].N > tasks[b.x].N; });
    if (!maps.empty())
      e = cudaMemcpy(maps_dev, maps.data(), sizeof(CUtensorMap) * maps.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && st.n_tasks)
      e = cudaMemcpy(st.gtasks_dev, tasks.data(), sizeof(GemmTask) * st.n_tasks, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && st.n_gjobs)
      e = cudaMemcpy(st.gjobs_dev, jobs.data(), sizeof(GemmJob) * st.n_gjobs, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && st.n_tiles)
      e = cudaMemcpy(st.tiles_dev, tiles.data(), sizeof(uint2) * st.n_tiles, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_commit upload");
  }
  p->committed = true;
  ctx->err[0] = 0;
  return Q4K_OK;
}

int q4k_plan_run(q4k_plan* p, void* stream) {
  if (!p) return Q4K_ERR_INVALID_ARG;
  q4k_ctx* ctx = p->ctx;
  if (!p->committed) return ctx_fail(ctx, Q4K_ERR_INVALID_ARG, "plan not committed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->gemm) {
    for (const Stage& st : p->stages) {
      cudaError_t e = launch_gemm_prep(st.gjobs_dev, st.n_gjobs, p->batch, p->parts, st.gjob_max_n,
                                       st.gjobs_aligned, ctx->device, s);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_run GEMM activation prep launch");
      e = launch_gemm_tasks(st.gtasks_dev, st.tiles_dev, st.n_tiles, p->parts, gemm_tile_tokens(p->parts, p->batch),
                            (uint32_t)ctx->sm_count, ctx->device, ctx->select.status, ctx->select.spin_limit, s);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_run GEMM launch");
    }
    ctx->err[0] = 0;
    return Q4K_OK;
  }
  for (const Stage& st : p->stages) {
    if (st.n_jobs && !st.prep) {
      JobList jl{};
      jl.dev = st.jobs_dev;
      jl.n = st.n_jobs;
      cudaError_t e = launch_xprep(jl, p->batch, s);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_run activation prep launch");
    }
    if (st.total_items) {
      TaskList tl{};
      tl.dev = st.tasks_dev;
      tl.sched = st.sched_dev;
      tl.grid = st.grid;
      tl.n = st.n_tasks;
      tl.total_items = st.total_items;
      tl.total_cost = st.total_cost;
      tl.select_task = st.select_task;
      tl.jobs = st.jobs_dev;
      tl.prep = st.prep ? 1u : 0u;
      tl.ksplit = st.ksplit;
      tl.fmt = st.fmt;
      tl.pairs = st.pairs ? 1u : 0u;
      cudaError_t e = launch_engine(tl, kNoMap, p->batch, !st.selects.empty(), ctx->select, ctx->sm_count, s);
      if (e != cudaSuccess) return ctx_cuda(ctx, e, "q4k_plan_run engine launch");
    }
  }
  ctx->err[0] = 0;
  return Q4K_OK;
}

int q4k_plan_launches(const q4k_plan* p) {
  if (!p || !p->committed) return -1;
  int n = 0;
  if (p->gemm) {
    for (const Stage& st : p->stages) n += (st.n_gjobs ? 1 : 0) + (st.n_tiles ? 1 : 0);
    return n;
  }
  for (const Stage& st : p->stages) n += (st.n_jobs && !st.prep ? 1 : 0) + (st.total_items ? 1 : 0);
  return n;
}

}  // extern "C"
