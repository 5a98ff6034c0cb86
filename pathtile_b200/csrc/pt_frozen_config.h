// pt_frozen_config.h -- launch configuration per path and intensity class, frozen offline.
//
// Written by `python -m pathtile_b200.pathtile --mode aggregate --write-header`:
// per path and per arithmetic-intensity class (in-range FMAs per output
// element: light < 12 <= medium < 24 <= heavy), the candidate (rows per tile,
// ring stages, CTAs per SM, threads per row) with the minimum sum of mean latency over that
// class's tuning shapes, ties to the smaller candidate -- the reference's
// selection rule (scripts/aggregate_pathtile_results.py:222-240) applied per
// class.  Deployment looks the class up; it does no per-shape search.
#pragma once

namespace pt {

struct LaunchCfg {
  int rows;         // rows per tile = threads doing math per CTA (32..256)
  int stages;       // shared-memory ring depth (2..4)
  int ctas_per_sm;  // persistent CTAs per SM (1..4), clamped by occupancy
  int tpr;          // consumer threads per row (1 or 2)
};

// kFrozenCfg[path][class]: path PT_PATH_FWD/DX/DK, class light/medium/heavy.
constexpr LaunchCfg kFrozenCfg[3][3] = {
    {{128, 3, 2, 1}, {128, 3, 2, 1}, {128, 3, 2, 1}},  // FWD: light, medium, heavy
    {{128, 3, 2, 1}, {128, 3, 2, 1}, {128, 3, 2, 1}},  // DX: light, medium, heavy
    {{256, 3, 1, 1}, {256, 3, 1, 1}, {256, 3, 1, 1}},  // DK: light, medium, heavy
};

// kFrozenEngine[path][class]: PT_ENGINE_FFMA (0) or PT_ENGINE_TENSOR (1); the
// tensor engine only ever applies to FWD/DX at L % 4 == 0.
constexpr int kFrozenEngine[3][3] = {
    {1, 1, 1},  // FWD: light, medium, heavy
    {1, 1, 1},  // DX: light, medium, heavy
    {0, 0, 0},  // DK: light, medium, heavy
};

// kFrozenBwd[class]: the kernel pt_dx_dk runs (PT_BWD_*) and the most channels
// a helper CTA of the tensor-core fused kernel may own (0: no helpers).
struct BwdChoice {
  int kernel;
  int helper_channels;
};
constexpr BwdChoice kFrozenBwd[3] = {
    {3, 0},  // light
    {3, 0},  // medium
    {3, 0},  // heavy
};

constexpr const char* kFrozenCfgSource = "B200 sweep of preset pathtile-train (2 trials x 3 visits), global policy per path";

}  // namespace pt
