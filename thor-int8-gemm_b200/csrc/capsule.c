/*
 * CPython entry point behind the `_C.cutlass_int8_dequant` proxy (patch_int8.py).
 *
 * comfy-kitchen calls `_C.cutlass_int8_dequant(x, w, x_scale, w_scale, bias, out, dtype_code,
 * stream)` with six DLPack capsules and a raw cudaStream_t (src/ck_int8_patch_thor.py:143-157).
 * This module reads the capsules' DLTensor descriptions in place -- no torch tensor is built
 * from them and they are not consumed, so the caller may still hand them to the stock
 * kernel -- applies the eligibility rules of the CUTLASS path the reference mirrors (:148-156)
 * and launches t8g_gemm_i8_dequant on `stream`.
 *
 *   cutlass_int8_dequant(x, w, x_scale, w_scale, bias, out, stream) -> True | None
 *     True: the GEMM was launched.  None: the call is not one this fast path takes (an
 *     argument that is not a DLPack capsule, a stream that is not an integer, or a call the
 *     eligibility rules decline); the caller then takes its general path.
 *     RuntimeError: the library rejected an eligible call (message from t8g_last_error).
 */
#define PY_SSIZE_T_CLEAN
#include <Python.h>
#include <stdint.h>

#include "../../include/thor_int8_gemm_b200.h"

/* The DLPack ABI (the dmlc/dlpack specification), the parts read here. */
typedef struct {
  int32_t device_type;
  int32_t device_id;
} DLDevice;
typedef struct {
  uint8_t code;
  uint8_t bits;
  uint16_t lanes;
} DLDataType;
typedef struct {
  void* data;
  DLDevice device;
  int32_t ndim;
  DLDataType dtype;
  int64_t* shape;
  int64_t* strides;
  uint64_t byte_offset;
} DLTensor;
typedef struct DLManagedTensor {
  DLTensor dl_tensor;
  void* manager_ctx;
  void (*deleter)(struct DLManagedTensor*);
} DLManagedTensor;
typedef struct {
  uint32_t major;
  uint32_t minor;
} DLPackVersion;
typedef struct DLManagedTensorVersioned {
  DLPackVersion version;
  void* manager_ctx;
  void (*deleter)(struct DLManagedTensorVersioned*);
  uint64_t flags;
  DLTensor dl_tensor;
} DLManagedTensorVersioned;

enum { kDLCUDA = 2 };
enum { kDLInt = 0, kDLFloat = 2, kDLBfloat = 4 };

#define MIN_M 128 /* src/ck_int8_patch_thor.py:30 */

static const DLTensor* dl_of(PyObject* o) {
  if (!PyCapsule_CheckExact(o)) return NULL;
  if (PyCapsule_IsValid(o, "dltensor")) {
    DLManagedTensor* m = (DLManagedTensor*)PyCapsule_GetPointer(o, "dltensor");
    return m ? &m->dl_tensor : NULL;
  }
  if (PyCapsule_IsValid(o, "dltensor_versioned")) {
    DLManagedTensorVersioned* m = (DLManagedTensorVersioned*)PyCapsule_GetPointer(o, "dltensor_versioned");
    return (m && m->version.major == 1) ? &m->dl_tensor : NULL;
  }
  return NULL;
}

static int is_type(const DLTensor* t, int code, int bits) {
  return t->dtype.code == code && t->dtype.bits == bits && t->dtype.lanes == 1;
}

static int64_t numel(const DLTensor* t) {
  int64_t n = 1;
  for (int i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}

/* Row-major compact (torch's is_contiguous: size-1 dimensions may carry any stride). */
static int contiguous(const DLTensor* t) {
  if (!t->strides) return 1;
  int64_t expect = 1;
  for (int i = t->ndim - 1; i >= 0; --i) {
    if (t->shape[i] != 1 && t->strides[i] != expect) return 0;
    expect *= t->shape[i];
  }
  return 1;
}

static void* ptr(const DLTensor* t) { return (char*)t->data + t->byte_offset; }

static PyObject* cutlass_int8_dequant(PyObject* self, PyObject* const* args, Py_ssize_t nargs) {
  (void)self;
  if (nargs != 7) {
    PyErr_SetString(PyExc_TypeError, "cutlass_int8_dequant(x, w, x_scale, w_scale, bias, out, stream)");
    return NULL;
  }
  const DLTensor* t[6];
  for (int i = 0; i < 6; ++i) {
    t[i] = dl_of(args[i]);
    if (!t[i]) Py_RETURN_NONE;
  }
  const DLTensor *x = t[0], *w = t[1], *xs = t[2], *ws = t[3], *b = t[4], *out = t[5];
  if (!PyLong_Check(args[6])) Py_RETURN_NONE;
  void* stream = PyLong_AsVoidPtr(args[6]);
  if (PyErr_Occurred()) {
    PyErr_Clear();
    Py_RETURN_NONE;
  }
  const int dev = x->device.device_id;
  for (int i = 0; i < 6; ++i)
    if (t[i]->device.device_type != kDLCUDA || t[i]->device.device_id != dev) Py_RETURN_NONE;
  if (x->ndim != 2 || w->ndim != 2 || out->ndim != 2) Py_RETURN_NONE;
  const int64_t M = x->shape[0], K = x->shape[1], N = w->shape[0];
  int out_code;
  if (is_type(out, kDLBfloat, 16))
    out_code = T8G_OUT_BF16;
  else if (is_type(out, kDLFloat, 16))
    out_code = T8G_OUT_F16;
  else if (is_type(out, kDLFloat, 32))
    out_code = T8G_OUT_F32;
  else
    Py_RETURN_NONE;
  const int64_t nb = numel(b), nws = numel(ws);
  /* the eligibility rules of the path the reference mirrors (src/ck_int8_patch_thor.py:148-156) */
  if (M < MIN_M || K % 16 || !contiguous(x) || !contiguous(w) || !contiguous(out) || !is_type(x, kDLInt, 8) ||
      !is_type(w, kDLInt, 8) || w->shape[1] != K || out->shape[0] != M || out->shape[1] != N ||
      !is_type(xs, kDLFloat, 32) || numel(xs) != M || !contiguous(xs) || !is_type(ws, kDLFloat, 32) ||
      (nws != 1 && nws != N) || !contiguous(ws) || (nb != 0 && nb != N) ||
      (nb && (b->dtype.code != out->dtype.code || b->dtype.bits != out->dtype.bits || !contiguous(b))))
    Py_RETURN_NONE;
  int prev = -1, rc = t8g_get_device(&prev);
  if (rc == T8G_OK && prev != dev) rc = t8g_set_device(dev);
  if (rc == T8G_OK)
    rc = t8g_gemm_i8_dequant(ptr(x), ptr(w), (const float*)ptr(xs), (const float*)ptr(ws), nws, nb ? ptr(b) : NULL,
                             nb, ptr(out), out_code, M, N, K, K, K, N, stream);
  if (prev >= 0 && prev != dev) {
    const int rc2 = t8g_set_device(prev);
    if (rc == T8G_OK) rc = rc2;
  }
  if (rc != T8G_OK) {
    PyErr_Format(PyExc_RuntimeError, "thor_int8_gemm_b200 error %d: %s", rc, t8g_last_error());
    return NULL;
  }
  Py_RETURN_TRUE;
}

static PyMethodDef methods[] = {
    {"cutlass_int8_dequant", (PyCFunction)(void (*)(void))cutlass_int8_dequant, METH_FASTCALL,
     "Launch the int8 fused-dequant GEMM from comfy-kitchen's DLPack capsules (True), or None."},
    {NULL, NULL, 0, NULL}};

static struct PyModuleDef module = {PyModuleDef_HEAD_INIT, "_t8g_capsule", NULL, -1, methods};

PyMODINIT_FUNC PyInit__t8g_capsule(void) { return PyModule_Create(&module); }
