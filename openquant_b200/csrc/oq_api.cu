// Error state, version and device queries of the openquant_b200 C ABI.
#include "oq_sm100.cuh"

#include <map>
#include <mutex>
#include <unordered_map>
#include <vector>

namespace oq {

namespace {
thread_local std::string g_last_error;

void vset(const char *fmt, va_list ap) {
    char buf[1024];
    vsnprintf(buf, sizeof(buf), fmt, ap);
    g_last_error = buf;
}
}  // namespace

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vset(fmt, ap);
    va_end(ap);
}

void clear_error() { g_last_error.clear(); }

int invalid(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vset(fmt, ap);
    va_end(ap);
    return OQ_ERR_INVALID;
}

int check_launch(const char *what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        set_error("%s: kernel launch failed: %s", what, cudaGetErrorString(err));
        return OQ_ERR_CUDA;
    }
    return OQ_OK;
}

int allow_dynamic_smem(const void *kern, size_t bytes) {
    static std::mutex mu;
    static std::map<std::pair<const void *, int>, size_t> done;
    int dev = 0;
    OQ_CUDA(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    auto it = done.find({kern, dev});
    if (it != done.end() && it->second >= bytes) return OQ_OK;
    OQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    done[{kern, dev}] = bytes;
    return OQ_OK;
}

int sm_count() {
    static std::mutex mu;
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

namespace {
std::mutex g_reader_mu;
std::vector<DeviceErrorReader> &readers() {
    static std::vector<DeviceErrorReader> v;
    return v;
}
}  // namespace

void register_device_error_reader(DeviceErrorReader fn) {
    std::lock_guard<std::mutex> lock(g_reader_mu);
    readers().push_back(fn);
}

namespace {
// Encoded maps by their arguments: a decode step re-launches on the same
// weights, and a map depends on nothing but these arguments, so a cached map
// is the one the encoder would return.
struct MapKey {
    const void *base;
    int dtype, esize, swizzle;
    uint64_t inner, outer, pitch;
    uint32_t box_inner, box_outer;
    bool operator==(const MapKey &o) const {
        return base == o.base && dtype == o.dtype && esize == o.esize && swizzle == o.swizzle && inner == o.inner &&
               outer == o.outer && pitch == o.pitch && box_inner == o.box_inner && box_outer == o.box_outer;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        uint64_t h = reinterpret_cast<uintptr_t>(k.base) * 0x9E3779B97F4A7C15ull;
        for (uint64_t v : {(uint64_t)k.dtype, (uint64_t)k.esize, (uint64_t)k.swizzle, k.inner, k.outer, k.pitch,
                           (uint64_t)k.box_inner, (uint64_t)k.box_outer})
            h = (h ^ v) * 0x100000001B3ull;
        return (size_t)h;
    }
};
constexpr size_t kMapCacheEntries = 1024;
}  // namespace

int make_tensor_map_2d(CUtensorMap *map, const void *base, CUtensorMapDataType dtype, int esize, uint64_t inner,
                       uint64_t outer, uint64_t pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                       CUtensorMapSwizzle swizzle) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::mutex mu;
    static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    if (!aligned(base, 16) || pitch_bytes % 16 != 0 || (uint64_t)box_inner * esize % 16 != 0) {
        set_error("tensor map: base, pitch and box row must be 16-byte multiples");
        return OQ_ERR_INVALID;
    }
    const MapKey key{base, (int)dtype, esize, (int)swizzle, inner, outer, pitch_bytes, box_inner, box_outer};
    std::lock_guard<std::mutex> lock(mu);
    auto hit = cache.find(key);
    if (hit != cache.end()) {
        *map = hit->second;
        return OQ_OK;
    }
    if (encode == nullptr) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
            set_error("cuTensorMapEncodeTiled unavailable (driver too old?)");
            return OQ_ERR_UNSUPPORTED;
        }
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {pitch_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (code %d)", (int)r);
        return OQ_ERR_CUDA;
    }
    if (cache.size() >= kMapCacheEntries) cache.clear();
    cache.emplace(key, *map);
    return OQ_OK;
}

}  // namespace oq

extern "C" int oq_take_device_error(int32_t *code) {
    oq::clear_error();
    if (code == nullptr) return oq::invalid("null pointer argument");
    *code = 0;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        oq::set_error("cudaDeviceSynchronize failed: %s", cudaGetErrorString(e));
        return OQ_ERR_CUDA;
    }
    std::vector<oq::DeviceErrorReader> rs;
    {
        std::lock_guard<std::mutex> lock(oq::g_reader_mu);
        rs = oq::readers();
    }
    int c = 0;
    for (auto fn : rs) {
        if (fn(&c) != OQ_OK) {
            oq::set_error("reading the device error word failed");
            return OQ_ERR_CUDA;
        }
    }
    *code = c;
    return OQ_OK;
}

extern "C" const char *oq_version(void) { return "openquant_b200 0.1.0 sm_100a"; }

extern "C" const char *oq_last_error(void) { return oq::g_last_error.c_str(); }

extern "C" int oq_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    int count = 0;
    for (int d = 0; d < n; ++d) {
        int major = 0;
        if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) == cudaSuccess && major == 10)
            ++count;
    }
    return count;
}
