// pt_frozen_config.h -- launch configuration per path, frozen offline.
//
// The B200 counterpart of the reference's frozen per-architecture constants
// (WARPS_PER_BLOCK / BWDK_BLOCK substituted into CUDA_TEMPLATE,
// kernels/warp_tiled_ampere.py:668-672, chosen by the argmin of summed latency
// over the 20 tuning shapes, scripts/aggregate_pathtile_results.py:222-240).
// Candidate axes here: rows per tile (one thread per row), TMA ring depth,
// and persistent CTAs per SM.  Deployment does no per-shape search.
#pragma once

namespace pt {

struct LaunchCfg {
  int rows;         // rows per tile = threads doing math per CTA (32..256)
  int stages;       // shared-memory ring depth (2..4)
  int ctas_per_sm;  // persistent CTAs per SM (1..4), clamped by occupancy
};

// Index: PT_PATH_FWD, PT_PATH_DX, PT_PATH_DK.
constexpr LaunchCfg kFrozenCfg[3] = {
    {128, 4, 2},  // FWD
    {128, 4, 2},  // DX
    {256, 3, 1},  // DK
};

// Provenance of the table above, reported by pt_config callers.
constexpr const char* kFrozenCfgSource = "B200 sweep of preset pathtile-train (3 trials)";

}  // namespace pt
