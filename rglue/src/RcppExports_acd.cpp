// RcppExports_acd.cpp — the registration glue for rglue/src/TensorAcd.cpp, in
// the form Rcpp::compileAttributes() writes into acediaR's
// src/RcppExports.cpp (see its entries at src/RcppExports.cpp:900-935 and the
// CallEntries table at 982-1071).  Running compileAttributes() on a tree that
// contains TensorAcd.cpp regenerates exactly these wrappers; they are kept
// here so the entry points are visible without R.
//
// When merging by hand: the wrappers of tensor_argmax_axis, tensor_argmin_axis,
// tensor_var_axis, tensor_to_dtype_unified, rand_tensor, rnorm_tensor and
// set_random_seed already exist in src/RcppExports.cpp (their definitions move
// from TensorReduction.cpp / TensorDataAccess.cpp / TensorRandom.cpp to
// TensorAcd.cpp); only the four new functions need wrappers and CallEntries
// lines.
//
// Not compiled here: R and Rcpp are absent from the build image.
#include <Rcpp.h>

using namespace Rcpp;

// tensor_softmax_axis_unified
SEXP tensor_softmax_axis_unified(SEXP tensor_ptr, int axis);
RcppExport SEXP _acediaR_tensor_softmax_axis_unified(SEXP tensor_ptrSEXP, SEXP axisSEXP) {
BEGIN_RCPP
    Rcpp::RObject rcpp_result_gen;
    Rcpp::RNGScope rcpp_rngScope_gen;
    Rcpp::traits::input_parameter< SEXP >::type tensor_ptr(tensor_ptrSEXP);
    Rcpp::traits::input_parameter< int >::type axis(axisSEXP);
    rcpp_result_gen = Rcpp::wrap(tensor_softmax_axis_unified(tensor_ptr, axis));
    return rcpp_result_gen;
END_RCPP
}
// tensor_cumsum_axis_unified
SEXP tensor_cumsum_axis_unified(SEXP tensor_ptr, int axis);
RcppExport SEXP _acediaR_tensor_cumsum_axis_unified(SEXP tensor_ptrSEXP, SEXP axisSEXP) {
BEGIN_RCPP
    Rcpp::RObject rcpp_result_gen;
    Rcpp::RNGScope rcpp_rngScope_gen;
    Rcpp::traits::input_parameter< SEXP >::type tensor_ptr(tensor_ptrSEXP);
    Rcpp::traits::input_parameter< int >::type axis(axisSEXP);
    rcpp_result_gen = Rcpp::wrap(tensor_cumsum_axis_unified(tensor_ptr, axis));
    return rcpp_result_gen;
END_RCPP
}
// tensor_cumprod_axis_unified
SEXP tensor_cumprod_axis_unified(SEXP tensor_ptr, int axis);
RcppExport SEXP _acediaR_tensor_cumprod_axis_unified(SEXP tensor_ptrSEXP, SEXP axisSEXP) {
BEGIN_RCPP
    Rcpp::RObject rcpp_result_gen;
    Rcpp::RNGScope rcpp_rngScope_gen;
    Rcpp::traits::input_parameter< SEXP >::type tensor_ptr(tensor_ptrSEXP);
    Rcpp::traits::input_parameter< int >::type axis(axisSEXP);
    rcpp_result_gen = Rcpp::wrap(tensor_cumprod_axis_unified(tensor_ptr, axis));
    return rcpp_result_gen;
END_RCPP
}
// tensor_compare_bool_unified
SEXP tensor_compare_bool_unified(SEXP a_ptr, SEXP b_ptr, std::string op);
RcppExport SEXP _acediaR_tensor_compare_bool_unified(SEXP a_ptrSEXP, SEXP b_ptrSEXP, SEXP opSEXP) {
BEGIN_RCPP
    Rcpp::RObject rcpp_result_gen;
    Rcpp::RNGScope rcpp_rngScope_gen;
    Rcpp::traits::input_parameter< SEXP >::type a_ptr(a_ptrSEXP);
    Rcpp::traits::input_parameter< SEXP >::type b_ptr(b_ptrSEXP);
    Rcpp::traits::input_parameter< std::string >::type op(opSEXP);
    rcpp_result_gen = Rcpp::wrap(tensor_compare_bool_unified(a_ptr, b_ptr, op));
    return rcpp_result_gen;
END_RCPP
}

// Lines for the CallEntries table of R_init_acediaR (src/RcppExports.cpp:982-1071):
//    {"_acediaR_tensor_softmax_axis_unified", (DL_FUNC) &_acediaR_tensor_softmax_axis_unified, 2},
//    {"_acediaR_tensor_cumsum_axis_unified", (DL_FUNC) &_acediaR_tensor_cumsum_axis_unified, 2},
//    {"_acediaR_tensor_cumprod_axis_unified", (DL_FUNC) &_acediaR_tensor_cumprod_axis_unified, 2},
//    {"_acediaR_tensor_compare_bool_unified", (DL_FUNC) &_acediaR_tensor_compare_bool_unified, 3},
