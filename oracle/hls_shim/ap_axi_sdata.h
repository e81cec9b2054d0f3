/* Minimal AXI-Stream side-channel struct for the reference's partitioned
 * native model. TEST INFRASTRUCTURE ONLY (oracle/Makefile). Fields the
 * reference uses: data, keep, strb, last (c_impl/gdn_model.cpp:5479-5700). */
#ifndef GDN_SHIM_AP_AXI_SDATA_H
#define GDN_SHIM_AP_AXI_SDATA_H

#include "ap_int.h"

template <int D, int U, int TI, int TD> struct ap_axiu {
    ap_uint<D> data;
    ap_uint<(D + 7) / 8> keep;
    ap_uint<(D + 7) / 8> strb;
    ap_uint<(U > 0 ? U : 1)> user;
    ap_uint<1> last;
    ap_uint<(TI > 0 ? TI : 1)> id;
    ap_uint<(TD > 0 ? TD : 1)> dest;
};

#endif
