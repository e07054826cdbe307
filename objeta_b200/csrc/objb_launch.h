// objb_launch.h -- host-side planning of the pipelined row-streaming kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace objb {

// Mirror of dev::RowLayout (same field order; the device struct is passed by
// value as a kernel argument).
struct RowLayoutHost {
  int rows, cols;
  int nblocks;
  int row_bytes;
  int srow_bytes;
  int nseg;
  int lpr;
  int rpw;
  int ngrp;
  int tstage;
  int nslots;
  int stage_bytes;
};

struct DeviceProps {
  int sm_count = 0;
  int max_smem_optin = 0;
  size_t l2_bytes = 0;
  int cc_major = 0, cc_minor = 0;
};

// Cached per-device properties (queried once per device).
int device_props(int device, DeviceProps* out);
int current_device(int* dev);

// Plans the row streaming of a rows x cols matrix whose packed rows are
// `row_bytes` (+ `srow_bytes` of split scales) long, with lane tiles covering
// `blocks_per_lane` blocks.  `dual` doubles the per-stage bytes (two matrices
// per stage).  Returns false when the shape cannot use the bulk-copy path.
// `smem_budget` bounds the stage ring: plain GEMVs (one matrix per call, calls
// back to back) keep the default; the MoE and FFN programs take the larger
// budget, where a third stage of wide rows shortens each expert's ramp.
constexpr int kGemvSmemBudget = 200 * 1024;
constexpr int kMoeSmemBudget = 226 * 1024;
bool plan_rows(int rows, int cols, int row_bytes, int srow_bytes, int blocks_per_lane, bool dual,
               int max_consumer_warps, RowLayoutHost* L, int smem_budget = kGemvSmemBudget);
// The same with the lanes a row spreads over given directly.
bool plan_rows_lanes(int rows, int cols, int row_bytes, int srow_bytes, int lanes, bool dual, int max_consumer_warps,
                     RowLayoutHost* L, int smem_budget = kGemvSmemBudget);

size_t pipe_smem_bytes(const RowLayoutHost& L);

// Opts a kernel into large dynamic shared memory once per (kernel, device).
int ensure_smem_attr_ptr(const void* kernel, int device, size_t bytes);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace objb
