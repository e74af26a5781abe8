// Instantiates one part of the kernels of one kernel_m: SC_KM (1..6) and
// SC_PART (0 = wide kernels, 1 = narrow kernels) are set by the build, so the
// instantiation sets compile in parallel.
#include "sc_kernels.cuh"

#ifndef SC_KM
#error "SC_KM must be defined (1..6)"
#endif
#ifndef SC_PART
#error "SC_PART must be defined (0 wide, 1 narrow)"
#endif

#define SC_CAT2(a, b) a##b
#define SC_CAT(a, b) SC_CAT2(a, b)

#if SC_PART == 0
sc::WideFn SC_CAT(sc_wide_kernel_km, SC_KM)(int vec, bool batch) {
  if (batch) {
    switch (vec) {
      case 1: return sc::spmm_wide_kernel<SC_KM, 1, true>;
      case 2: return sc::spmm_wide_kernel<SC_KM, 2, true>;
      default: return sc::spmm_wide_kernel<SC_KM, 4, true>;
    }
  }
  switch (vec) {
    case 1: return sc::spmm_wide_kernel<SC_KM, 1, false>;
    case 2: return sc::spmm_wide_kernel<SC_KM, 2, false>;
    default: return sc::spmm_wide_kernel<SC_KM, 4, false>;
  }
}
#else
template <int VT>
static sc::NarrowFn narrow_of(int nb) {
  if constexpr (VT == 4) {
    switch (nb) {
      case 1: return sc::spmm_lane_kernel<SC_KM, 1>;
      case 2: return sc::spmm_lane_kernel<SC_KM, 2>;
      default: return sc::spmm_lane_kernel<SC_KM, 4>;
    }
  } else {
    switch (nb) {
      case 1: return sc::spmm_narrow_kernel<SC_KM, 1, VT>;
      case 2: return sc::spmm_narrow_kernel<SC_KM, 2, VT>;
      default: return sc::spmm_narrow_kernel<SC_KM, 4, VT>;
    }
  }
}

sc::LaneXFn SC_CAT(sc_lane_x_kernel_km, SC_KM)(int nb) {
  (void)nb;  // SpMV only (N = 2 staged measured no faster than split blocks)
  return sc::spmm_lane_x_kernel<SC_KM, 1>;
}

// vt: 0 = fp32 records, 1 = fp16 compact records, 2 = bf16 compact records,
// 3 = split blocks (16-bit columns, fp32 values), 4 = lane blocks
sc::NarrowFn SC_CAT(sc_narrow_kernel_km, SC_KM)(int nb, int vt) {
  switch (vt) {
    case 1: return narrow_of<1>(nb);
    case 2: return narrow_of<2>(nb);
    case 3: return narrow_of<3>(nb);
    case 4: return narrow_of<4>(nb);
    default: return narrow_of<0>(nb);
  }
}
#endif
