# gpuTensor_acd.R — R wrappers of acediaR over the entry points in
# rglue/src/TensorAcd.cpp.  They replace the functions of R/gpuTensor.R named
# below; everything else in R/gpuTensor.R is unchanged.
#
# Not run here: R is absent from the build image.  The same semantics are
# implemented and tested by the Python mirror (acedia-r_b200/acediar/tensor.py:
# softmax, cumsum, cumprod, argmax, argmin, var, compare, to_dtype).

# softmax (R/gpuTensor.R:1718): the whole tensor as before, or along `axis`
# (1-based), the row softmax exp(v - max(v)) / sum(exp(v - max(v))).
softmax <- function(x, axis = NULL) {
  if (!inherits(x, "gpuTensor")) stop("Object is not a gpuTensor")
  if (is.null(axis)) return(tensor_softmax_unified(x))
  if (!is.numeric(axis) || length(axis) != 1 || axis < 1 || axis > length(shape(x)))
    stop("axis must be a single positive integer within tensor dimensions")
  tensor_softmax_axis_unified(x, as.integer(axis - 1L))
}

# cumsum / cumprod (R/gpuTensor.R:2234-2277): the flattened column-major
# vector as before (now on the device), or along `axis`.
cumsum.gpuTensor <- function(x, axis = NULL) {
  if (!inherits(x, "gpuTensor")) stop("Object is not a gpuTensor")
  if (is.null(axis)) return(tensor_cumsum_axis_unified(x, -1L))
  if (!is.numeric(axis) || length(axis) != 1 || axis < 1 || axis > length(shape(x)))
    stop("axis must be a single positive integer within tensor dimensions")
  tensor_cumsum_axis_unified(x, as.integer(axis - 1L))
}

cumprod.gpuTensor <- function(x, axis = NULL) {
  if (!inherits(x, "gpuTensor")) stop("Object is not a gpuTensor")
  if (is.null(axis)) return(tensor_cumprod_axis_unified(x, -1L))
  if (!is.numeric(axis) || length(axis) != 1 || axis < 1 || axis > length(shape(x)))
    stop("axis must be a single positive integer within tensor dimensions")
  tensor_cumprod_axis_unified(x, as.integer(axis - 1L))
}

# argmax / argmin with an axis (R/gpuTensor.R:1942-1979): tensor_argmax_axis
# now computes on the device (it was a stub that stopped with "not yet
# implemented").  Indices come back 0-based int64, as TensorWrapper::argmax
# defines them; R's are 1-based, added here as R/gpuTensor.R:1749-1754 does.
.one_based <- function(res) {
  arr <- as.array(res) + 1
  gpu_tensor(as.vector(arr), shape(res), dtype = "int64")
}

argmax.gpuTensor <- function(x, axis = NULL, keep.dims = FALSE, ...) {
  if (!inherits(x, "gpuTensor")) stop("Object is not a gpuTensor")
  if (is.null(axis)) return(tensor_argmax_unified(x))
  if (!is.numeric(axis) || length(axis) != 1 || axis < 1 || axis > length(shape(x)))
    stop("axis must be within dimensions of tensor")
  .one_based(tensor_argmax_axis(x, as.integer(axis - 1L), keep.dims))
}

argmin.gpuTensor <- function(x, axis = NULL, keep.dims = FALSE, ...) {
  if (!inherits(x, "gpuTensor")) stop("Object is not a gpuTensor")
  if (is.null(axis)) return(tensor_argmin_unified(x))
  if (!is.numeric(axis) || length(axis) != 1 || axis < 1 || axis > length(shape(x)))
    stop("axis must be within dimensions of tensor")
  .one_based(tensor_argmin_axis(x, as.integer(axis - 1L), keep.dims))
}

# Comparisons with a bool result (one byte per element, values 0/1).  The
# operators `>`, `<`, `==` of R/gpuTensor.R keep the reference's 0/1 in the
# input dtype; compare() gives the bool form, and `!=`, `>=`, `<=` become one
# kernel each instead of the reference's composites (R/gpuTensor.R:1872-1930).
compare <- function(a, b, op = c("gt", "lt", "eq", "ne", "ge", "le")) {
  op <- match.arg(op)
  if (!inherits(a, "gpuTensor") || !inherits(b, "gpuTensor")) stop("Both operands must be gpuTensor objects")
  tensor_compare_bool_unified(a, b, op)
}
