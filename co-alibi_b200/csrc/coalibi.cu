// C-ABI entry points of libcoalibi_sm100.so (declared in include/coalibi.h):
// argument validation, TMA tensor-map encoding and kernel dispatch.  Nothing
// here allocates device memory or synchronises.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "coalibi.h"
#include "ctx_guard.h"
#include "fwd.cuh"
#include "decode.cuh"
#include "bwd.cuh"

namespace coalibi {

// Human-readable detail of the last failure on this thread (coalibi_last_error()).
static thread_local char g_last_error[256] = "";

void set_last_error_detail(const char* msg) { snprintf(g_last_error, sizeof(g_last_error), "%s", msg); }

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 3-D view (D, rows, heads) of a contiguous [.., heads, rows, D] 16-bit tensor,
// loaded as boxes of 64 columns x box_rows rows with the 128-byte swizzle the
// UMMA descriptors expect.  Rows past `rows` read as zero.
int make_tmap(CUtensorMap* map, const void* base, int D, int rows, int heads, int box_rows, bool bf16) {
  auto fn = encode_fn();
  if (fn == nullptr) {
    snprintf(g_last_error, sizeof(g_last_error), "cuTensorMapEncodeTiled unavailable from the driver");
    return COALIBI_ERR_TENSOR_MAP;
  }
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)rows, (cuuint64_t)heads};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)rows * D * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    snprintf(g_last_error, sizeof(g_last_error),
             "cuTensorMapEncodeTiled -> %d (base=%p D=%d rows=%d heads=%d box_rows=%d map=%p)", (int)r, base, D,
             rows, heads, box_rows, (void*)map);
    return COALIBI_ERR_TENSOR_MAP;
  }
  return COALIBI_OK;
}

// Driver entry points used to bind and restore contexts.  Binding goes through
// the driver API so that the runtime's per-thread device selection (what
// cudaSetDevice changes) is never touched: a thread that had no context current
// still has none afterwards, and one that had selected device 0 still has.
struct DrvFns {
  PFN_cuCtxGetCurrent_v4000 ctx_get = nullptr;
  PFN_cuCtxSetCurrent_v4000 ctx_set = nullptr;
  PFN_cuCtxGetDevice_v2000 ctx_device = nullptr;
  PFN_cuDeviceGet_v2000 device_get = nullptr;
  PFN_cuDevicePrimaryCtxRetain_v7000 primary_retain = nullptr;
  PFN_cuPointerGetAttributes_v7000 ptr_attrs = nullptr;
  bool ok = false;
};

template <typename F>
static void load_entry(const char* name, F& fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
    fn = reinterpret_cast<F>(p);
}

static const DrvFns& drv() {
  static DrvFns f;
  static std::once_flag once;
  std::call_once(once, [] {
    load_entry("cuCtxGetCurrent", f.ctx_get);
    load_entry("cuCtxSetCurrent", f.ctx_set);
    load_entry("cuCtxGetDevice", f.ctx_device);
    load_entry("cuDeviceGet", f.device_get);
    load_entry("cuDevicePrimaryCtxRetain", f.primary_retain);
    load_entry("cuPointerGetAttributes", f.ptr_attrs);
    f.ok = f.ctx_get && f.ctx_set && f.ctx_device && f.device_get && f.primary_retain && f.ptr_attrs;
  });
  return f;
}

CtxGuard::CtxGuard() {
  const DrvFns& f = drv();
  if (f.ok) saved_ok_ = f.ctx_get(&saved_) == CUDA_SUCCESS;
}

CtxGuard::~CtxGuard() {
  if (!saved_ok_) return;
  const DrvFns& f = drv();
  CUcontext now = nullptr;
  if (f.ctx_get(&now) == CUDA_SUCCESS && now == saved_) return;
  f.ctx_set(saved_);
}

namespace {

constexpr int kMaxDevices = 64;
constexpr unsigned kDefaultTimeoutMs = 2000;

// Per-device one-time setup: architecture check and opt-in shared memory sizes.
struct DeviceState {
  std::once_flag once;
  int status = COALIBI_ERR_DEVICE;
  int sm_count = 0;
};
DeviceState g_dev[kMaxDevices];

template <typename K>
bool set_smem(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
}

// Primary context of each device, retained once and kept for the life of the
// process (as the runtime keeps it).
struct PrimaryCtx {
  std::once_flag once;
  CUcontext ctx = nullptr;
};
PrimaryCtx g_primary[kMaxDevices];

// Make a context of the device that owns `ptr` current on the calling thread: the
// caller's own context when it is already on that device, else the device's
// primary context (the one the runtime and PyTorch use).  Callers such as
// autograd's backward worker threads may reach us with no context current, which
// the tensor-map encoder rejects.  The entry point's CtxGuard undoes the switch.
int bind_device(const void* ptr) {
  const DrvFns& f = drv();
  if (!f.ok) {
    snprintf(g_last_error, sizeof(g_last_error), "CUDA driver entry points unavailable");
    return COALIBI_ERR_DEVICE;
  }
  CUpointer_attribute names[3] = {CU_POINTER_ATTRIBUTE_MEMORY_TYPE, CU_POINTER_ATTRIBUTE_DEVICE_ORDINAL,
                                  CU_POINTER_ATTRIBUTE_IS_MANAGED};
  unsigned int mem_type = 0;
  int ordinal = -1;
  unsigned int managed = 0;
  void* vals[3] = {&mem_type, &ordinal, &managed};
  if (f.ptr_attrs(3, names, vals, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    snprintf(g_last_error, sizeof(g_last_error), "cuPointerGetAttributes failed for %p", ptr);
    return COALIBI_ERR_DEVICE;
  }
  if ((mem_type != CU_MEMORYTYPE_DEVICE && !managed) || ordinal < 0 || ordinal >= kMaxDevices) {
    snprintf(g_last_error, sizeof(g_last_error), "%p is not device memory", ptr);
    return COALIBI_ERR_DEVICE;
  }
  CUcontext cur = nullptr;
  CUdevice cur_dev = -1;
  if (f.ctx_get(&cur) == CUDA_SUCCESS && cur != nullptr && f.ctx_device(&cur_dev) == CUDA_SUCCESS) {
    CUdevice want = -1;
    if (f.device_get(&want, ordinal) == CUDA_SUCCESS && want == cur_dev) return COALIBI_OK;
  }
  PrimaryCtx& pc = g_primary[ordinal];
  std::call_once(pc.once, [&pc, &f, ordinal] {
    CUdevice d;
    CUcontext c = nullptr;
    if (f.device_get(&d, ordinal) == CUDA_SUCCESS && f.primary_retain(&c, d) == CUDA_SUCCESS) pc.ctx = c;
  });
  if (pc.ctx == nullptr || f.ctx_set(pc.ctx) != CUDA_SUCCESS) {
    snprintf(g_last_error, sizeof(g_last_error), "cannot make device %d's primary context current", ordinal);
    return COALIBI_ERR_DEVICE;
  }
  return COALIBI_OK;
}

int device_setup(const void* ptr) {
  if (int rc = bind_device(ptr)) return rc;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return COALIBI_ERR_DEVICE;
  DeviceState& st = g_dev[dev];
  std::call_once(st.once, [&st, dev] {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0) {
      st.status = COALIBI_ERR_DEVICE;
      return;
    }
    if (cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        st.sm_count <= 0) {
      st.status = COALIBI_ERR_DEVICE;
      return;
    }
    bool ok = true;
    ok &= set_smem(coalibi_fwd_kernel<128, false>, FwdLayout<128>::ALLOC);
    ok &= set_smem(coalibi_fwd_kernel<128, true>, FwdLayout<128>::ALLOC);
    ok &= set_smem(coalibi_fwd_kernel<64, false>, FwdLayout<64>::ALLOC);
    ok &= set_smem(coalibi_fwd_kernel<64, true>, FwdLayout<64>::ALLOC);
    ok &= set_smem(coalibi_decode_mma_kernel<128, false, 32>, DecodeMmaSmem<128, 32>::BYTES);
    ok &= set_smem(coalibi_decode_mma_kernel<128, true, 32>, DecodeMmaSmem<128, 32>::BYTES);
    ok &= set_smem(coalibi_decode_mma_kernel<128, false, 16>, DecodeMmaSmem<128, 16>::BYTES);
    ok &= set_smem(coalibi_decode_mma_kernel<128, true, 16>, DecodeMmaSmem<128, 16>::BYTES);
    ok &= set_smem(coalibi_decode_mma_kernel<64, false, 16>, DecodeMmaSmem<64, 16>::BYTES);
    ok &= set_smem(coalibi_decode_mma_kernel<64, true, 16>, DecodeMmaSmem<64, 16>::BYTES);
    ok &= bwd_set_smem_attributes();
    st.status = ok ? COALIBI_OK : COALIBI_ERR_LAUNCH;
  });
  return st.status;
}

}  // namespace

int enter_device(const void* ptr, void* stream) {
  if (int rc = device_setup(ptr)) return rc;
  int dev = -1, sdev = -1;
  cudaGetDevice(&dev);
  if (cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev) != cudaSuccess) {
    cudaGetLastError();
    snprintf(g_last_error, sizeof(g_last_error), "cudaStreamGetDevice failed for stream %p", stream);
    return COALIBI_ERR_DEVICE;
  }
  if (sdev != dev) {
    snprintf(g_last_error, sizeof(g_last_error),
             "stream %p belongs to device %d but the tensors are on device %d", stream, sdev, dev);
    return COALIBI_ERR_DEVICE;
  }
  return COALIBI_OK;
}

namespace {

// SM count of the current device (device_setup has run for it)
int current_sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  return g_dev[dev].sm_count;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

int check_common(int B, int Hq, int Hkv, int Sq, int Skv, int D, int dtype, int slopes_dtype) {
  if (D != 64 && D != 128) return COALIBI_ERR_HEAD_DIM;
  if (dtype != COALIBI_F16 && dtype != COALIBI_BF16) return COALIBI_ERR_DTYPE;
  if (slopes_dtype != COALIBI_F16 && slopes_dtype != COALIBI_BF16 && slopes_dtype != COALIBI_F32)
    return COALIBI_ERR_DTYPE;
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Skv <= 0) return COALIBI_ERR_SHAPE;
  if (Hq % Hkv != 0) return COALIBI_ERR_SHAPE;
  const long long nq = (Sq + 127) / 128;
  if ((long long)B * Hq * nq > 0x7fffffffLL) return COALIBI_ERR_SHAPE;
  if ((long long)B * Hq > 0x7fffffffLL || (long long)B * Hkv * Skv > (1LL << 40)) return COALIBI_ERR_SHAPE;
  return COALIBI_OK;
}

namespace {

unsigned long long timeout_ns(unsigned ms) {
  return (unsigned long long)(ms == 0 ? kDefaultTimeoutMs : ms) * 1000000ull;
}

template <int D, bool BF16>
int launch_fwd_impl(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const FwdParams& p,
               cudaStream_t stream) {
  // Large problems: persistent, one CTA per SM walking (head, query tile) items in a
  // static snake order (the next item's loads and first MMAs overlap this one's
  // epilogue).  Below about 12 items per SM the static order leaves SMs idle at the
  // end, so each CTA then takes one item and the hardware balances (measured:
  // B = 1, 2 at H16 S4096 one-item 25% faster; B = 4, 8 persistent 2-4% faster).
  const int n_items = p.B * p.Hq * p.n_qtiles;
  const int sms = current_sm_count();
  const int grid = (n_items >= 12 * sms) ? sms : n_items;
  cudaError_t e = launch_pdl(coalibi_fwd_kernel<D, BF16>, dim3(grid), dim3(FwdLayout<D>::THREADS), FwdLayout<D>::ALLOC,
                             stream, tq, tk, tv, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(g_last_error, sizeof(g_last_error), "forward launch: %s", cudaGetErrorString(e));
    return COALIBI_ERR_LAUNCH;
  }
  return COALIBI_OK;
}

template <int D, bool BF16>
int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const FwdParams& p,
               cudaStream_t stream) {
  return launch_fwd_impl<D, BF16>(tq, tk, tv, p, stream);
}

}  // namespace
}  // namespace coalibi

namespace coalibi {
namespace {
// Warps wait on barriers nothing arrives on: the first to time out raises the
// abort flag and the status word; the others see the flag and return too.
__global__ void __launch_bounds__(64) selftest_wait_kernel(int* status, unsigned long long timeout_ns) {
  __shared__ uint64_t bar[2];
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  CtaGuard g{&abort_flag, status, timeout_ns};
  mbar_wait(&bar[threadIdx.x >> 5], 0, g);
}
}  // namespace
}  // namespace coalibi

using namespace coalibi;

extern "C" int coalibi_selftest_wait_timeout(unsigned int timeout_ms, int* status, void* stream) {
  if (status == nullptr) return COALIBI_ERR_NULL_POINTER;
  CtxGuard guard;
  if (int rc = enter_device(status, stream)) return rc;
  selftest_wait_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(status, timeout_ns(timeout_ms));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    snprintf(g_last_error, sizeof(g_last_error), "self-test launch: %s", cudaGetErrorString(e));
    return COALIBI_ERR_LAUNCH;
  }
  return COALIBI_OK;
}

extern "C" int coalibi_fwd(const CoalibiFwdArgs* a, void* stream) {
  if (a == nullptr) return COALIBI_ERR_NULL_POINTER;
  if (!a->q || !a->k || !a->v || !a->o || !a->lse || !a->rowsig || !a->slopes) return COALIBI_ERR_NULL_POINTER;
  int rc = check_common(a->B, a->Hq, a->Hkv, a->Sq, a->Skv, a->D, a->dtype, a->slopes_dtype);
  if (rc) return rc;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o)) return COALIBI_ERR_ALIGNMENT;
  CtxGuard guard;
  if ((rc = enter_device(a->q, stream))) return rc;
  const bool bf16 = a->dtype == COALIBI_BF16;
  CUtensorMap tq, tk, tv;
  if ((rc = make_tmap(&tq, a->q, a->D, a->Sq, a->B * a->Hq, 128, bf16))) return rc;
  if ((rc = make_tmap(&tk, a->k, a->D, a->Skv, a->B * a->Hkv, 128, bf16))) return rc;
  if ((rc = make_tmap(&tv, a->v, a->D, a->Skv, a->B * a->Hkv, 128, bf16))) return rc;
  FwdParams p{};
  p.o = a->o;
  p.lse = a->lse;
  p.rowsig = a->rowsig;
  p.slopes = a->slopes;
  p.B = a->B;
  p.Hq = a->Hq;
  p.Hkv = a->Hkv;
  p.Sq = a->Sq;
  p.Skv = a->Skv;
  p.slopes_dtype = a->slopes_dtype;
  p.causal = a->causal ? 1 : 0;
  p.sm_scale = a->sm_scale;
  p.status = a->status;
  p.timeout_ns = timeout_ns(a->timeout_ms);
  p.n_qtiles = (a->Sq + 127) / 128;
  p.n_kvtiles = (a->Skv + 127) / 128;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->D == 128) return bf16 ? launch_fwd<128, true>(tq, tk, tv, p, s) : launch_fwd<128, false>(tq, tk, tv, p, s);
  return bf16 ? launch_fwd<64, true>(tq, tk, tv, p, s) : launch_fwd<64, false>(tq, tk, tv, p, s);
}

namespace coalibi {
namespace {
template <int D, bool BF16>
int launch_decode(const DecodeParams& p, cudaStream_t stream) {
  const dim3 grid_p(p.B * p.Hkv, p.n_chunks / 4, p.n_rgroups);
  // 16-key warp steps halve the shared memory (three CTAs per SM instead of one at
  // D = 128): faster at D = 64 and when several row groups re-read K and V from L2;
  // one row group at D = 128 streams K and V at ~5 TB/s with 32-key steps
  // (measured: B8 Hq32 Hkv8 Skv32768 0.213 vs 0.225 ms; Sq16 Skv131072 0.414 vs
  // 0.322 ms; D64 B16 H12 Skv4096 0.052 vs 0.045 ms).
  if (D == 64 || p.n_rgroups > 1)
    coalibi_decode_mma_kernel<D, BF16, 16><<<grid_p, 128, DecodeMmaSmem<D, 16>::BYTES, stream>>>(p);
  else
    coalibi_decode_mma_kernel<D, BF16, 32><<<grid_p, 128, DecodeMmaSmem<D, 32>::BYTES, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    coalibi_decode_combine_kernel<D, BF16><<<p.B * p.Hq * p.Sq, D, 0, stream>>>(p);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    snprintf(g_last_error, sizeof(g_last_error), "decode launch: %s", cudaGetErrorString(e));
    return COALIBI_ERR_LAUNCH;
  }
  return COALIBI_OK;
}
}  // namespace
}  // namespace coalibi

extern "C" size_t coalibi_fwd_decode_workspace_bytes(int B, int Hq, int Hkv, int Sq, int Skv, int D) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || Skv <= 0 || Hq % Hkv != 0 || Sq > kDecodeMaxSq) return 0;
  if (D != 64 && D != 128) return 0;
  return D == 128 ? decode_plan<128>(B, Hq, Hkv, Sq, Skv).bytes : decode_plan<64>(B, Hq, Hkv, Sq, Skv).bytes;
}

extern "C" int coalibi_fwd_decode(const CoalibiFwdArgs* a, void* workspace, size_t workspace_bytes, void* stream) {
  if (a == nullptr) return COALIBI_ERR_NULL_POINTER;
  if (!a->q || !a->k || !a->v || !a->o || !a->lse || !a->rowsig || !a->slopes) return COALIBI_ERR_NULL_POINTER;
  int rc = check_common(a->B, a->Hq, a->Hkv, a->Sq, a->Skv, a->D, a->dtype, a->slopes_dtype);
  if (rc) return rc;
  if (a->Sq > kDecodeMaxSq) return COALIBI_ERR_SHAPE;
  if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->o)) return COALIBI_ERR_ALIGNMENT;
  const size_t need = coalibi_fwd_decode_workspace_bytes(a->B, a->Hq, a->Hkv, a->Sq, a->Skv, a->D);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) return COALIBI_ERR_WORKSPACE;
  CtxGuard guard;
  if ((rc = enter_device(a->q, stream))) return rc;
  DecodeParams p{};
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.slopes = a->slopes;
  p.o = a->o;
  p.lse = a->lse;
  p.rowsig = a->rowsig;
  p.ws = static_cast<float*>(workspace);
  p.B = a->B;
  p.Hq = a->Hq;
  p.Hkv = a->Hkv;
  p.Sq = a->Sq;
  p.Skv = a->Skv;
  p.slopes_dtype = a->slopes_dtype;
  p.causal = a->causal ? 1 : 0;
  p.sm_scale = a->sm_scale;
  const DecodePlan pl = a->D == 128 ? decode_plan<128>(a->B, a->Hq, a->Hkv, a->Sq, a->Skv)
                                    : decode_plan<64>(a->B, a->Hq, a->Hkv, a->Sq, a->Skv);
  p.n_chunks = pl.records;
  p.chunk_keys = pl.chunk_keys;
  p.n_rgroups = pl.n_rgroups;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16 = a->dtype == COALIBI_BF16;
  if (a->D == 128) return bf16 ? launch_decode<128, true>(p, s) : launch_decode<128, false>(p, s);
  return bf16 ? launch_decode<64, true>(p, s) : launch_decode<64, false>(p, s);
}

extern "C" size_t coalibi_bwd_workspace_bytes(int B, int Hq, int Hkv, int Sq, int Skv, int D) {
  (void)Hkv;
  (void)D;
  if (B <= 0 || Hq <= 0 || Sq <= 0 || Skv <= 0) return 0;
  // enough for either mask (the non-causal problem has every tile visible)
  const size_t c = bwd_workspace_preferred(B, Hq, Sq, Skv, true);
  const size_t n = bwd_workspace_preferred(B, Hq, Sq, Skv, false);
  return c > n ? c : n;
}

extern "C" size_t coalibi_bwd_workspace_size(const CoalibiBwdArgs* a) {
  if (a == nullptr || a->B <= 0 || a->Hq <= 0 || a->Sq <= 0 || a->Skv <= 0) return 0;
  return bwd_workspace_preferred(a->B, a->Hq, a->Sq, a->Skv, a->causal != 0);
}

extern "C" size_t coalibi_bwd_workspace_min_bytes(int B, int Hq, int Hkv, int Sq, int Skv, int D) {
  (void)Hkv;
  (void)D;
  if (B <= 0 || Hq <= 0 || Sq <= 0 || Skv <= 0) return 0;
  return bwd_workspace_recompute(B, Hq, Sq, Skv).total;
}

extern "C" int coalibi_bwd_phases(const CoalibiBwdArgs* a, int phase_mask, void* stream) {
  if (a == nullptr) return COALIBI_ERR_NULL_POINTER;
  if (phase_mask & ~7) return COALIBI_ERR_SHAPE;
  if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->rowsig || !a->slopes || !a->dq || !a->dk ||
      !a->dv)
    return COALIBI_ERR_NULL_POINTER;
  int rc = check_common(a->B, a->Hq, a->Hkv, a->Sq, a->Skv, a->D, a->dtype, a->slopes_dtype);
  if (rc) return rc;
  const void* ptrs[8] = {a->q, a->k, a->v, a->o, a->dout, a->dq, a->dk, a->dv};
  for (const void* ptr : ptrs)
    if (!aligned16(ptr)) return COALIBI_ERR_ALIGNMENT;
  const BwdWorkspace ws = bwd_workspace_for(a->B, a->Hq, a->Sq, a->Skv, a->causal != 0, a->workspace_bytes);
  if (a->workspace == nullptr || ws.total == 0) return COALIBI_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0) return COALIBI_ERR_ALIGNMENT;
  CtxGuard guard;
  if ((rc = enter_device(a->q, stream))) return rc;
  return bwd_launch(*a, ws, timeout_ns(a->timeout_ms), static_cast<cudaStream_t>(stream), phase_mask);
}

extern "C" int coalibi_bwd(const CoalibiBwdArgs* a, void* stream) { return coalibi_bwd_phases(a, 7, stream); }

extern "C" int coalibi_bwd_carry(const CoalibiBwdArgs* a, const float* dA_carry_in, void* stream) {
  if (a == nullptr || dA_carry_in == nullptr) return COALIBI_ERR_NULL_POINTER;
  if (!a->q || !a->k || !a->v || !a->o || !a->dout || !a->lse || !a->rowsig || !a->slopes || !a->dq || !a->dk ||
      !a->dv)
    return COALIBI_ERR_NULL_POINTER;
  int rc = check_common(a->B, a->Hq, a->Hkv, a->Sq, a->Skv, a->D, a->dtype, a->slopes_dtype);
  if (rc) return rc;
  const void* ptrs[8] = {a->q, a->k, a->v, a->o, a->dout, a->dq, a->dk, a->dv};
  for (const void* ptr : ptrs)
    if (!aligned16(ptr)) return COALIBI_ERR_ALIGNMENT;
  const BwdWorkspace ws = bwd_workspace_for(a->B, a->Hq, a->Sq, a->Skv, a->causal != 0, a->workspace_bytes);
  if (a->workspace == nullptr || ws.total == 0) return COALIBI_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(a->workspace) & 255u) != 0) return COALIBI_ERR_ALIGNMENT;
  CtxGuard guard;
  if ((rc = enter_device(a->q, stream))) return rc;
  return bwd_launch(*a, ws, timeout_ns(a->timeout_ms), static_cast<cudaStream_t>(stream), 7, dA_carry_in);
}

extern "C" int coalibi_describe_launch(int which, int B, int Hq, int Hkv, int Sq, int Skv, int D, int causal,
                                       int device, char* buf, size_t buf_len) {
  if (buf == nullptr || buf_len == 0) return COALIBI_ERR_NULL_POINTER;
  buf[0] = '\0';
  CtxGuard guard;
  if (int rc = check_common(B, Hq, Hkv, Sq, Skv, D, COALIBI_F16, COALIBI_F32)) return rc;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0) {
    cudaGetLastError();
    return COALIBI_ERR_DEVICE;
  }
  const int nq = (Sq + 127) / 128;
  if (which == 0) {
    // the rule of launch_fwd_impl
    const long long items = (long long)B * Hq * nq;
    const bool persistent = items >= 12LL * sms;
    const int threads = D == 128 ? FwdLayout<128>::THREADS : FwdLayout<64>::THREADS;
    const int smem = D == 128 ? FwdLayout<128>::ALLOC : FwdLayout<64>::ALLOC;
    snprintf(buf, buf_len,
             "forward coalibi_fwd_kernel<D=%d>: %s grid of %lld CTAs over %lld (head, 128-row query tile) items, "
             "%d threads, %d B shared memory, 128-key tiles",
             D, persistent ? "persistent (one CTA per SM, snake order)" : "one item per CTA",
             persistent ? (long long)sms : items, items, threads, smem);
    return COALIBI_OK;
  }
  if (which == 1) {
    if (Sq > kDecodeMaxSq) return COALIBI_ERR_SHAPE;
    const DecodePlan pl = D == 128 ? decode_plan<128>(B, Hq, Hkv, Sq, Skv) : decode_plan<64>(B, Hq, Hkv, Sq, Skv);
    const int step = (D == 64 || pl.n_rgroups > 1) ? 16 : 32;  // the rule of launch_decode
    snprintf(buf, buf_len,
             "decode coalibi_decode_mma_kernel<D=%d, %d-key steps>: grid (%d, %d, %d) of 128 threads, %d keys per "
             "CTA chunk, %d row groups; then coalibi_decode_combine_kernel over %lld query rows",
             D, step, B * Hkv, pl.records / 4, pl.n_rgroups, pl.chunk_keys, pl.n_rgroups, (long long)B * Hq * Sq);
    return COALIBI_OK;
  }
  if (which == 2) {
    const BwdWorkspace st = bwd_workspace_stored(B, Hq, Sq, Skv, causal != 0);
    const bool stored = bwd_workspace_preferred(B, Hq, Sq, Skv, causal != 0) == st.total;
    const int athreads = D == 128 ? BwdALayout<128>::THREADS : BwdALayout<64>::THREADS;
    if (stored) {
      snprintf(buf, buf_len,
               "backward, stored path (P / dS scratch %.1f MB): coalibi_bwd_delta_kernel<D=%d>; "
               "coalibi_bwd_a_kernel<D=%d, stores P and dS> (query-major) grid %lld x %d threads; "
               "coalibi_bwd_kv_kernel<D=%d> (streaming dV = P^T dO, dK = dS^T Q, GQA group of %d heads summed in "
               "TMEM) grid %lld x %d threads",
               (double)(st.total - st.p_off) / 1e6, D, D, (long long)B * Hq * nq, athreads, D, Hq / Hkv,
               (long long)B * Hkv * ((Skv + 127) / 128), D == 128 ? BwdKVLayout<128>::THREADS : BwdKVLayout<64>::THREADS);
    } else {
      const int kb = D == 128 ? BwdB128Layout::KB : BwdBLayout<64>::KB;
      const long long nb = (Skv + kb - 1) / kb;
      snprintf(buf, buf_len,
               "backward, recompute path (P / dS scratch would exceed the cap): coalibi_bwd_delta_kernel<D=%d>; "
               "coalibi_bwd_a_kernel<D=%d> (query-major, carries every 32 keys) grid %lld x %d threads; %s "
               "(key-major, recomputes S, dP, P, dS; %d keys per CTA, GQA group of %d heads summed in TMEM) grid "
               "%lld x %d threads",
               D, D, (long long)B * Hq * nq, athreads,
               D == 128 ? "coalibi_bwd_b128_kernel" : "coalibi_bwd_b_kernel<D=64>", kb, Hq / Hkv,
               (long long)B * Hkv * nb, D == 128 ? BwdB128Layout::THREADS : BwdBLayout<64>::THREADS);
    }
    return COALIBI_OK;
  }
  return COALIBI_ERR_SHAPE;
}

extern "C" const char* coalibi_strerror(int code) {
  switch (code) {
    case COALIBI_OK: return "ok";
    case COALIBI_ERR_NULL_POINTER: return "null pointer argument";
    case COALIBI_ERR_HEAD_DIM: return "unsupported head dim (expected 64 or 128)";
    case COALIBI_ERR_DTYPE: return "unsupported dtype (expected float16 or bfloat16)";
    case COALIBI_ERR_SHAPE: return "invalid shape (non-positive size, Hq % Hkv != 0, or too large)";
    case COALIBI_ERR_ALIGNMENT: return "pointer not 16-byte aligned (workspace: 256-byte)";
    case COALIBI_ERR_LAUNCH: return "CUDA kernel launch failed";
    case COALIBI_ERR_TENSOR_MAP: return "TMA tensor map encoding failed";
    case COALIBI_ERR_WORKSPACE: return "backward workspace missing or too small";
    case COALIBI_ERR_DEVICE: return "current CUDA device is not an sm_100 (B200) GPU";
    case COALIBI_ERR_TIMEOUT: return "a bounded in-kernel wait timed out";
    default: return "unknown error";
  }
}

extern "C" int coalibi_abi_version(void) { return COALIBI_ABI_VERSION; }

extern "C" const char* coalibi_last_error(void) { return g_last_error; }
