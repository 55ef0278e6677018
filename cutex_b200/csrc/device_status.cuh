// Device-side error reporting shared by every kernel of the library: one
// status word (the first error wins) and, in builds compiled with
// -DCUTEX_CHECKED, consistency checks on the indices each kernel derives
// (tile coordinates, TMEM column ranges, store extents, workspace slots).
//
// A failed check never faults and never traps: it records its site code and
// the offending value, and the caller skips the access and leaves its role's
// loop; the other roles then stop at their bounded waits. The host reads the
// status word with cutex_last_device_status (CUTEX_ERR_DEVICE_CHECK for codes
// from 0x200) and the site and value with cutex_device_check_record. Without
// CUTEX_CHECKED every check is the constant `true` and compiles to nothing.
#pragma once

#include <cstdint>

namespace cutex {

// The library is a single translation unit, so the header defines these.
__device__ int g_cutex_device_status = 0;
// {site code, offending value} of the failed check that set the status word.
__device__ long long g_cutex_check_record[2] = {0, 0};

enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutProducer = 0x101,
  kDevTimeoutMma = 0x102,
  kDevTimeoutEpilogue = 0x103,
  kDevTimeoutAccEmpty = 0x104,
  kDevTimeoutScheduler = 0x105,
  kDevTimeoutQuantize = 0x106,  // columnwise quantiser: a TMA tile never arrived
  kDevBadTile = 0x201,  // a scheduled tile id outside [0, num_tiles): work stopped, nothing accessed
  // Checked builds only:
  kChkTile = 0x211,          // GEMM tile coordinates outside the output tile grid
  kChkTmemCols = 0x212,      // a TMEM column range outside the CTA's allocation
  kChkStore = 0x213,         // an output store outside D's padded extent
  kChkScaleOffset = 0x214,   // a scale-byte offset outside the scale array
  kChkSkinnySegment = 0x215, // a skinny segment outside [0, num_n_tiles) x [0, K / 128)
  kChkWorkspace = 0x216,     // a partial slot, contributor or counter index outside the workspace
  kChkCodeOffset = 0x217,    // a quantiser code store outside the code array
  kChkQuantTile = 0x218,     // a columnwise quantiser tile outside x
  kChkSelfTest = 0x21F,      // cutex_selftest_device_check
};

#ifdef CUTEX_CHECKED
constexpr bool kCheckedBuild = true;
#else
constexpr bool kCheckedBuild = false;
#endif

// True when `ok`. Otherwise (checked builds) records the failure: the thread
// that sets the status word stores the site and the value.
__device__ __forceinline__ bool dev_check(bool ok, int site, long long value) {
  if constexpr (!kCheckedBuild) {
    return true;
  } else {
    if (ok) return true;
    if (atomicCAS(&g_cutex_device_status, 0, site) == 0) {
      g_cutex_check_record[1] = value;
      g_cutex_check_record[0] = site;
    }
    return false;
  }
}

}  // namespace cutex
