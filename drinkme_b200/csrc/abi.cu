// The extern "C" entry points of libdrinkme_b200.so (declared in
// include/drinkme_b200.h): tensor load/free, the GEMV dispatch, decode, the
// gulp schedule, the raw GEMV and the device error word.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "dm_internal.h"

namespace dm {

void set_error(char *err, size_t len, const std::string &msg) {
    if (err && len) {
        size_t n = std::min(len - 1, msg.size());
        std::memcpy(err, msg.data(), n);
        err[n] = 0;
    }
}

}  // namespace dm

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int fail(char *err, size_t len, int code, const std::string &msg) {
    dm::set_error(err, len, msg);
    return code;
}

int cuda_fail(char *err, size_t len, cudaError_t e, const char *what) {
    return fail(err, len, DM_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

void free_tensor(dm_tensor *t) {
    if (!t) return;
    DeviceGuard g(t->device);
    if (t->d_data) cudaFree(t->d_data);
    if (t->d_unit16) cudaFree(t->d_unit16);
    if (t->d_rowdir) cudaFree(t->d_rowdir);
    if (t->S.partials) cudaFree(t->S.partials);
    if (t->S.counters) cudaFree(t->S.counters);
    if (t->S.xsplit) cudaFree(t->S.xsplit);
    if (t->S.err) cudaFree(t->S.err);
    delete t;
}

}  // namespace

extern "C" int dm_version(void) { return 100; }

namespace {

// A pack of another radix profile (gulp, balanced, ...) with whole
// 1024-weight blocks, re-encoded as sip: the loader decodes its rows to the
// exact bf16 bits and this library's encoder (dm_pack_plan/encode) packs
// them again with widths (3, 8), so the sip kernels serve it. The decoded
// weights are the same bits; the device bytes differ from the source pack's
// by a few percent. Returns false (serve the pack as given) when the profile
// is already sip, the blocks do not fit the sip kernels, or sip would take
// more than 5/4 of the source words.
struct Transcoded {
    std::vector<uint8_t> pal;
    std::vector<uint32_t> off, data;
    int32_t widths[2] = {3, 8};
};

bool transcode_to_sip(const dm::PackPart &P, Transcoded &o, dm::PackPart &out) {
    if (P.nw == 2 && P.widths[0] == 3 && P.widths[1] == 8) return false;
    if (P.B != 1024 || P.C % 1024 != 0) return false;
    const int64_t rows = P.row1 - P.row0, NB = P.C / 1024;
    std::vector<uint16_t> bits((size_t)(rows * P.C));
    dm::decode_rows(P, bits.data());
    o.pal.assign(7, 0);
    o.off.assign((size_t)(rows * NB + 1), 0);
    uint64_t nwords = 0;
    char e[256];
    if (dm_pack_plan(bits.data(), rows, P.C, o.widths, 2, 1024, 0, o.pal.data(), o.off.data(), &nwords, e,
                     sizeof e) != DM_OK)
        return false;
    int64_t src_words = 0;
    dm::pack_read_bytes(P, &src_words);
    if ((int64_t)nwords * 4 > src_words * 5) return false;
    o.data.assign((size_t)nwords, 0);
    if (dm_pack_encode(bits.data(), rows, P.C, o.widths, 2, 1024, 0, o.pal.data(), o.off.data(), o.data.data(),
                       nwords, e, sizeof e) != DM_OK)
        return false;
    out = dm::PackPart{o.pal.data(), o.pal.size(), o.off.data(), o.off.size(), o.data.data(), o.data.size(), rows,
                       P.C, o.widths, 2, 1024, 0, rows};
    return true;
}

// Lays `parts` out, copies the layout to `device` and sizes the scratch.
int create_from_parts(const dm::PackPart *given, int nparts, int32_t device, dm_tensor **out, char *err,
                      size_t err_len) {
    std::string msg;
    dm_tensor *t = new dm_tensor();
    t->device = device;
    std::string bytes, unit16, rowdir;
    // the source packs' own read bytes and payload words (the reference's count)
    int64_t src_read = 0, src_words = 0;
    for (int i = 0; i < nparts; ++i) {
        int64_t w = 0;
        src_read += dm::pack_read_bytes(given[i], &w);
        src_words += w;
    }
    std::vector<Transcoded> owned((size_t)nparts);
    std::vector<dm::PackPart> parts(given, given + nparts);
    bool transcoded = false;
    for (int i = 0; i < nparts; ++i) transcoded |= transcode_to_sip(given[i], owned[i], parts[i]);
    if (transcoded)
        for (int i = 0; i < nparts; ++i)
            if (!(parts[i].nw == 2 && parts[i].widths[0] == 3)) {  // all parts sip, or none re-encoded
                parts.assign(given, given + nparts);
                transcoded = false;
                break;
            }
    if (dm::build_layout(parts.data(), nparts, t->L, bytes, unit16, msg, &rowdir)) {
        delete t;
        return fail(err, err_len, DM_EINVAL, msg);
    }
    t->L.dev_read_bytes = t->L.read_bytes;
    if (transcoded) {
        t->L.src_nw = given[0].nw;
        for (int i = 0; i < given[0].nw; ++i) t->L.src_widths[i] = given[0].widths[i];
        t->L.read_bytes = src_read;
        t->L.payload_words = src_words;
        t->L.R = nparts == 1 ? given[0].R : t->L.R;
        t->L.row0 = nparts == 1 ? given[0].row0 : 0;
    }
    DeviceGuard g(device);
    cudaError_t e;
    cudaDeviceGetAttribute(&t->sms, cudaDevAttrMultiProcessorCount, device);
    if ((e = cudaMalloc(&t->d_data, bytes.size())) != cudaSuccess) {
        free_tensor(t);
        return cuda_fail(err, err_len, e, "cudaMalloc(layout)");
    }
    t->data_bytes = bytes.size();
    if ((e = cudaMalloc(&t->d_unit16, unit16.size())) != cudaSuccess) {
        free_tensor(t);
        return cuda_fail(err, err_len, e, "cudaMalloc(unit directory)");
    }
    if ((e = cudaMemcpy(t->d_data, bytes.data(), bytes.size(), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(t->d_unit16, unit16.data(), unit16.size(), cudaMemcpyHostToDevice)) != cudaSuccess) {
        free_tensor(t);
        return cuda_fail(err, err_len, e, "cudaMemcpy(layout)");
    }
    t->resident_bytes = bytes.size() + unit16.size();
    if (!rowdir.empty()) {
        if ((e = cudaMalloc(&t->d_rowdir, rowdir.size())) != cudaSuccess ||
            (e = cudaMemcpy(t->d_rowdir, rowdir.data(), rowdir.size(), cudaMemcpyHostToDevice)) != cudaSuccess) {
            free_tensor(t);
            return cuda_fail(err, err_len, e, "cudaMalloc(row directory)");
        }
        t->rowdir_bytes = rowdir.size();
        t->resident_bytes += rowdir.size();
    }
    if ((e = cudaMalloc(&t->S.err, sizeof(int))) != cudaSuccess || (e = cudaMemset(t->S.err, 0, sizeof(int))) != cudaSuccess) {
        free_tensor(t);
        return cuda_fail(err, err_len, e, "cudaMalloc(error word)");
    }
    if (t->L.fast_sip) {
        const int64_t workers = std::min<int64_t>((int64_t)t->sms, t->L.units);  // one per CTA
        t->S.max_workers = (int32_t)workers;
        const size_t pbytes = (size_t)workers * 2 * 128 * sizeof(float);
        const size_t cbytes = (size_t)t->L.tiles * sizeof(int);
        const size_t xbytes = (size_t)6 * (size_t)t->L.C * 2;
        if ((e = cudaMalloc(&t->S.partials, pbytes)) != cudaSuccess ||
            (e = cudaMalloc(&t->S.counters, cbytes)) != cudaSuccess ||
            (e = cudaMemset(t->S.counters, 0, cbytes)) != cudaSuccess ||
            (e = cudaMalloc(&t->S.xsplit, xbytes)) != cudaSuccess) {
            free_tensor(t);
            return cuda_fail(err, err_len, e, "cudaMalloc(scratch)");
        }
        t->resident_bytes += pbytes + cbytes + xbytes;
    }
    *out = t;
    return DM_OK;
}

int check_part(const dm_pack_part &p, const char *who, char *err, size_t err_len) {
    if (!p.host_offsets || !p.host_data || !p.host_widths || (!p.host_palette && p.npalette))
        return fail(err, err_len, DM_EINVAL, std::string(who) + ": null pointer");
    if (p.nwidths < 2 || p.nwidths > 8)
        return fail(err, err_len, DM_EINVAL, "radix needs 2..8 widths in 1..8, ending with the exponent width");
    std::string msg;
    if (dm::validate_pack(p.host_palette, p.npalette, p.host_offsets, p.noffsets, p.nwords, p.R, p.C, p.host_widths,
                          p.nwidths, p.block_size, msg))
        return fail(err, err_len, DM_EINVAL, msg);
    return DM_OK;
}

dm::PackPart to_part(const dm_pack_part &p) {
    return dm::PackPart{p.host_palette, p.npalette, p.host_offsets, p.noffsets, p.host_data, p.nwords, p.R, p.C,
                        p.host_widths, p.nwidths, p.block_size, p.row_begin, p.row_end};
}

}  // namespace

extern "C" int dm_tensor_create(const uint8_t *palette, size_t npalette, const uint32_t *offsets, size_t noffsets,
                                const uint32_t *data, size_t nwords, int64_t R, int64_t C, const int32_t *widths,
                                int32_t nwidths, int32_t block_size, int64_t row_begin, int64_t row_end,
                                int32_t device, dm_tensor **out, char *err, size_t err_len) {
    if (!out) return fail(err, err_len, DM_EINVAL, "dm_tensor_create: null pointer");
    *out = nullptr;
    const dm_pack_part p{palette, npalette, offsets, noffsets, data, nwords, R, C, widths, nwidths, block_size,
                         row_begin, row_end};
    if (int rc = check_part(p, "dm_tensor_create", err, err_len)) return rc;
    const dm::PackPart part = to_part(p);
    return create_from_parts(&part, 1, device, out, err, err_len);
}

extern "C" int dm_tensor_create_multi(const dm_pack_part *parts, int32_t nparts, int32_t device, dm_tensor **out,
                                      char *err, size_t err_len) {
    if (!out || !parts) return fail(err, err_len, DM_EINVAL, "dm_tensor_create_multi: null pointer");
    *out = nullptr;
    if (nparts < 1 || nparts > 64) return fail(err, err_len, DM_EINVAL, "dm_tensor_create_multi: 1..64 parts");
    std::vector<dm::PackPart> ps;
    for (int i = 0; i < nparts; ++i) {
        if (int rc = check_part(parts[i], "dm_tensor_create_multi", err, err_len)) return rc;
        ps.push_back(to_part(parts[i]));
    }
    return create_from_parts(ps.data(), nparts, device, out, err, err_len);
}

extern "C" int dm_tensor_clone(const dm_tensor *src, dm_tensor **out, char *err, size_t err_len) {
    if (!src || !out) return fail(err, err_len, DM_EINVAL, "dm_tensor_clone: null pointer");
    *out = nullptr;
    DeviceGuard g(src->device);
    dm_tensor *t = new dm_tensor();
    t->device = src->device;
    t->L = src->L;
    t->sms = src->sms;
    t->K = src->K;
    t->data_bytes = src->data_bytes;
    t->S.max_workers = src->S.max_workers;
    cudaError_t e;
    const size_t ubytes = (size_t)(src->L.units + 1) * sizeof(uint32_t);
    if ((e = cudaMalloc(&t->d_data, src->data_bytes)) != cudaSuccess ||
        (e = cudaMemcpy(t->d_data, src->d_data, src->data_bytes, cudaMemcpyDeviceToDevice)) != cudaSuccess ||
        (e = cudaMalloc(&t->d_unit16, ubytes)) != cudaSuccess ||
        (e = cudaMemcpy(t->d_unit16, src->d_unit16, ubytes, cudaMemcpyDeviceToDevice)) != cudaSuccess ||
        (e = cudaMalloc(&t->S.err, sizeof(int))) != cudaSuccess ||
        (e = cudaMemset(t->S.err, 0, sizeof(int))) != cudaSuccess) {
        free_tensor(t);
        return cuda_fail(err, err_len, e, "dm_tensor_clone");
    }
    t->resident_bytes = src->data_bytes + ubytes;
    if (src->d_rowdir) {
        if ((e = cudaMalloc(&t->d_rowdir, src->rowdir_bytes)) != cudaSuccess ||
            (e = cudaMemcpy(t->d_rowdir, src->d_rowdir, src->rowdir_bytes, cudaMemcpyDeviceToDevice)) != cudaSuccess) {
            free_tensor(t);
            return cuda_fail(err, err_len, e, "dm_tensor_clone(row directory)");
        }
        t->rowdir_bytes = src->rowdir_bytes;
        t->resident_bytes += src->rowdir_bytes;
    }
    if (src->L.fast_sip) {
        const size_t pbytes = (size_t)t->S.max_workers * 2 * 128 * sizeof(float);
        const size_t cbytes = (size_t)t->L.tiles * sizeof(int);
        const size_t xbytes = (size_t)6 * (size_t)t->L.C * 2;
        if ((e = cudaMalloc(&t->S.partials, pbytes)) != cudaSuccess ||
            (e = cudaMalloc(&t->S.counters, cbytes)) != cudaSuccess ||
            (e = cudaMemset(t->S.counters, 0, cbytes)) != cudaSuccess ||
            (e = cudaMalloc(&t->S.xsplit, xbytes)) != cudaSuccess) {
            free_tensor(t);
            return cuda_fail(err, err_len, e, "dm_tensor_clone(scratch)");
        }
        t->resident_bytes += pbytes + cbytes + xbytes;
    }
    *out = t;
    return DM_OK;
}

extern "C" int dm_tensor_destroy(dm_tensor *t) {
    free_tensor(t);
    return DM_OK;
}

extern "C" int dm_tensor_get_info(const dm_tensor *t, dm_tensor_info *info) {
    if (!t || !info) return DM_EINVAL;
    std::memset(info, 0, sizeof(*info));
    info->R = t->L.R;
    info->C = t->L.C;
    info->row_begin = t->L.row0;
    info->rows = t->L.rows;
    info->block_size = t->L.B;
    // the pack's own profile (a re-encoded pack reports the widths it came with)
    info->nwidths = t->L.src_nw ? t->L.src_nw : t->L.nw;
    for (int i = 0; i < 8; ++i) info->widths[i] = t->L.src_nw ? t->L.src_widths[i] : t->L.widths[i];
    info->device_bytes_per_call = t->L.src_nw ? t->L.dev_read_bytes : t->L.read_bytes;
    info->nblocks = t->L.rows * t->L.NB;
    info->payload_words = t->L.payload_words;
    info->read_bytes = t->L.read_bytes;
    info->resident_bytes = (int64_t)t->resident_bytes;
    info->fast_path = t->L.fast_sip ? 1 : 0;
    info->device = t->device;
    info->layout_ptr = reinterpret_cast<uint64_t>(t->d_data);
    info->layout_bytes = (int64_t)t->data_bytes;
    return DM_OK;
}

extern "C" int dm_gemv(const dm_tensor *t, const void *x, int32_t x_dtype, int64_t M, const void *bias, void *out,
                       int32_t out_dtype, void *stream, char *err, size_t err_len) {
    if (!t || !x || !out) return fail(err, err_len, DM_EINVAL, "dm_gemv: null pointer");
    if (M < 1 || M > DM_MC_MAX)
        return fail(err, err_len, DM_EINVAL,
                    "radix gemv_mc: M=" + std::to_string(M) + " outside 1.." + std::to_string(DM_MC_MAX));
    if ((x_dtype != DM_BF16 && x_dtype != DM_F32) || (out_dtype != DM_BF16 && out_dtype != DM_F32))
        return fail(err, err_len, DM_EINVAL, "dm_gemv: dtype must be DM_BF16 or DM_F32");
    if ((reinterpret_cast<uintptr_t>(x) & (x_dtype == DM_F32 ? 3u : 1u)) != 0)
        return fail(err, err_len, DM_EINVAL, "dm_gemv: activations not aligned to their element size");
    DeviceGuard g(t->device);
    std::string msg;
    const uint16_t *b16 = reinterpret_cast<const uint16_t *>(bias);
    const int of32 = out_dtype == DM_F32;
    // a sip tensor is served by the sip kernel at any activation alignment
    // (unaligned bf16 rows are copied to the tensor's staging buffer first);
    // the general kernel reads only plain-stream layouts
    const int rc = t->L.fast_sip
                       ? dm::gemv_sip_rows(t, x, x_dtype == DM_F32, M, b16, out, of32, t->S.xsplit, 6 * t->L.C,
                                           t->S.partials, t->S.counters, t->S.max_workers, stream, msg)
                       : dm::launch_gemv_generic(t, x, x_dtype == DM_F32, M, b16, out, of32, stream, msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_tensor_set_launch(dm_tensor *t, const dm_launch *l, char *err, size_t err_len) {
    if (!t || !l) return fail(err, err_len, DM_EINVAL, "dm_tensor_set_launch: null pointer");
    if (l->slots < 0 || l->slots > 6)
        return fail(err, err_len, DM_EINVAL, "dm_tensor_set_launch: slots must be 0 (measured rule) or 1..6");
    if (l->split < 0 || l->split > 2)
        return fail(err, err_len, DM_EINVAL, "dm_tensor_set_launch: split must be 0 (auto), 1 (stream-K) or 2 (tiles)");
    if (l->skew < -1 || l->skew > 64)
        return fail(err, err_len, DM_EINVAL, "dm_tensor_set_launch: skew must be -1 (default) or 0..64");
    if (l->resident < -1 || l->resident > 16)
        return fail(err, err_len, DM_EINVAL, "dm_tensor_set_launch: resident must be -1 (default) or 0..16");
    t->K.slots = l->slots;
    t->K.split = l->split;
    t->K.skew = l->skew;
    if (l->prefetch < -1 || l->prefetch > 32)
        return fail(err, err_len, DM_EINVAL, "dm_tensor_set_launch: prefetch must be -1 (default) or 0..32");
    t->K.resident = l->resident;
    t->K.prefetch = l->prefetch;
    return DM_OK;
}

extern "C" int dm_gemv_plan(const dm_tensor *t, int64_t M, int32_t x_dtype, dm_launch_plan *plan, char *err,
                            size_t err_len) {
    if (!t || !plan) return fail(err, err_len, DM_EINVAL, "dm_gemv_plan: null pointer");
    if (M < 1 || M > DM_MC_MAX)
        return fail(err, err_len, DM_EINVAL,
                    "radix gemv_mc: M=" + std::to_string(M) + " outside 1.." + std::to_string(DM_MC_MAX));
    if (!t->L.fast_sip) return fail(err, err_len, DM_EINVAL, "dm_gemv_plan: not a sip fast-path tensor");
    std::memset(plan, 0, sizeof(*plan));
    std::string msg;
    const int Mv = x_dtype == DM_F32 ? (int)(3 * std::min<int64_t>(2, M)) : (int)M;
    const int rc = dm::gemv_plan(t, Mv, plan, msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_decode(const dm_tensor *t, uint16_t *out, void *stream, char *err, size_t err_len) {
    if (!t || !out) return fail(err, err_len, DM_EINVAL, "dm_decode: null pointer");
    DeviceGuard g(t->device);
    std::string msg;
    int rc = t->L.fast_sip ? dm::launch_decode_sip(t, out, stream, msg) : dm::launch_decode_generic(t, out, stream, msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_decode_pack(const uint8_t *host_palette, size_t npalette, const uint32_t *host_offsets,
                              size_t noffsets, size_t nwords, int64_t R, int64_t C, const int32_t *host_widths,
                              int32_t nwidths, int32_t block_size, const uint32_t *d_data, const uint32_t *d_offsets,
                              uint16_t *d_out, void *stream, char *err, size_t err_len) {
    if (!host_palette || !host_offsets || !host_widths || !d_data || !d_offsets || !d_out)
        return fail(err, err_len, DM_EINVAL, "dm_decode_pack: null pointer");
    std::string msg;
    if (dm::validate_pack(host_palette, npalette, host_offsets, noffsets, nwords, R, C, host_widths, nwidths,
                          block_size, msg))
        return fail(err, err_len, DM_EINVAL, msg);
    int rc = dm::launch_decode_pack(host_palette, npalette, R, C, host_widths, nwidths, block_size, d_data, d_offsets,
                                    d_out, stream, msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_prepare_schedule(const uint32_t *data, size_t nwords, const uint32_t *offsets, int64_t C,
                                   const int32_t *widths, int32_t nwidths, int32_t block_size, int64_t nblocks,
                                   uint16_t *out, void *stream, char *err, size_t err_len) {
    if (!data || !offsets || !widths || !out) return fail(err, err_len, DM_EINVAL, "dm_prepare_schedule: null pointer");
    if (nwidths < 2 || nwidths > 8 || block_size < 32 || block_size > 4096 || C <= 0)
        return fail(err, err_len, DM_EINVAL, "dm_prepare_schedule: invalid parameters");
    std::string msg;
    int rc = dm::launch_prepare_schedule(data, nwords, offsets, C, widths, nwidths, block_size, nblocks, out, stream,
                                         msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_gemv_raw(const void *w, int64_t R, int64_t C, const void *x, int32_t x_dtype, int64_t M,
                           const void *bias, void *out, int32_t out_dtype, void *stream, char *err, size_t err_len) {
    if (!w || !x || !out) return fail(err, err_len, DM_EINVAL, "dm_gemv_raw: null pointer");
    if (M < 1 || M > DM_MC_MAX)
        return fail(err, err_len, DM_EINVAL,
                    "gemv_narrow: M=" + std::to_string(M) + " outside 1.." + std::to_string(DM_MC_MAX));
    if (R <= 0 || C <= 0) return fail(err, err_len, DM_EINVAL, "dm_gemv_raw: empty weight");
    if ((x_dtype != DM_BF16 && x_dtype != DM_F32) || (out_dtype != DM_BF16 && out_dtype != DM_F32))
        return fail(err, err_len, DM_EINVAL, "dm_gemv_raw: dtype must be DM_BF16 or DM_F32");
    if ((reinterpret_cast<uintptr_t>(w) & 1) || (reinterpret_cast<uintptr_t>(x) & (x_dtype == DM_F32 ? 3u : 1u)))
        return fail(err, err_len, DM_EINVAL, "dm_gemv_raw: weight or activations not aligned to their element size");
    std::string msg;
    int rc = dm::launch_gemv_raw(w, R, C, x, x_dtype == DM_F32, M, reinterpret_cast<const uint16_t *>(bias), out,
                                 out_dtype == DM_F32, stream, msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_tensor_check(const dm_tensor *t, int32_t *device_error, char *err, size_t err_len) {
    if (!t || !device_error) return fail(err, err_len, DM_EINVAL, "dm_tensor_check: null pointer");
    DeviceGuard g(t->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(err, err_len, e, "cudaDeviceSynchronize");
    int v = 0;
    if ((e = cudaMemcpy(&v, t->S.err, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(err, err_len, e, "cudaMemcpy(error word)");
    if (v && (e = cudaMemset(t->S.err, 0, sizeof(int))) != cudaSuccess)
        return cuda_fail(err, err_len, e, "cudaMemset(error word)");
    *device_error = v;
    return DM_OK;
}

extern "C" int dm_gemv_gather(const dm_tensor *t, const void *x, int64_t M, const void *bias, int32_t out_dtype,
                              const dm_gather *g, void *stream, char *err, size_t err_len) {
    if (!t || !x || !g) return fail(err, err_len, DM_EINVAL, "dm_gemv_gather: null pointer");
    if (M < 1 || M > DM_MC_MAX)
        return fail(err, err_len, DM_EINVAL,
                    "radix gemv_mc: M=" + std::to_string(M) + " outside 1.." + std::to_string(DM_MC_MAX));
    if (out_dtype != DM_BF16 && out_dtype != DM_F32)
        return fail(err, err_len, DM_EINVAL, "dm_gemv_gather: dtype must be DM_BF16 or DM_F32");
    if (!t->L.fast_sip) return fail(err, err_len, DM_EINVAL, "dm_gemv_gather: needs a sip tensor (the fast path)");
    if ((reinterpret_cast<uintptr_t>(x) & 15) != 0)
        return fail(err, err_len, DM_EINVAL, "dm_gemv_gather: activations must be 16-byte aligned");
    if (g->world < 1 || g->world > DM_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
        return fail(err, err_len, DM_EINVAL, "dm_gemv_gather: rank outside a world of 1.." + std::to_string(DM_MAX_RANKS));
    if (g->slot < t->L.rows) return fail(err, err_len, DM_EINVAL, "dm_gemv_gather: slot smaller than this rank's rows");
    for (int r = 0; r < g->world; ++r)
        if (!g->peer_out[r] || !g->peer_flags[r]) return fail(err, err_len, DM_EINVAL, "dm_gemv_gather: null peer pointer");
    if (!g->gen || !g->done || !g->abort || (!g->wait_flags) != (!g->wait_gen))
        return fail(err, err_len, DM_EINVAL, "dm_gemv_gather: counters / wait words incomplete");
    DeviceGuard guard(t->device);
    std::string msg;
    int rc = dm::launch_gemv_sip_with(t, reinterpret_cast<const uint16_t *>(x), t->L.C, (int)M, 1, (int)M,
                                      reinterpret_cast<const uint16_t *>(bias), nullptr, out_dtype == DM_F32,
                                      t->S.partials, t->S.counters, t->S.err, t->S.max_workers, stream, msg, g);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}

extern "C" int dm_ipc_handle(const void *dptr, uint8_t *out64, char *err, size_t err_len) {
    if (!dptr || !out64) return fail(err, err_len, DM_EINVAL, "dm_ipc_handle: null pointer");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void *>(dptr));
    if (e != cudaSuccess) return cuda_fail(err, err_len, e, "cudaIpcGetMemHandle");
    static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
    std::memcpy(out64, &h, 64);
    return DM_OK;
}

extern "C" int dm_ipc_open(const uint8_t *handle64, int32_t device, void **dptr, char *err, size_t err_len) {
    if (!handle64 || !dptr) return fail(err, err_len, DM_EINVAL, "dm_ipc_open: null pointer");
    DeviceGuard g(device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle64, 64);
    cudaError_t e = cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(err, err_len, e, "cudaIpcOpenMemHandle");
    return DM_OK;
}

extern "C" int dm_ipc_close(void *dptr, char *err, size_t err_len) {
    if (!dptr) return fail(err, err_len, DM_EINVAL, "dm_ipc_close: null pointer");
    cudaError_t e = cudaIpcCloseMemHandle(dptr);
    if (e != cudaSuccess) return cuda_fail(err, err_len, e, "cudaIpcCloseMemHandle");
    return DM_OK;
}

extern "C" int dm_device_alloc(int32_t device, size_t bytes, void **dptr, char *err, size_t err_len) {
    if (!dptr || bytes == 0) return fail(err, err_len, DM_EINVAL, "dm_device_alloc: null pointer or no bytes");
    DeviceGuard g(device);
    cudaError_t e = cudaMalloc(dptr, bytes);
    if (e != cudaSuccess) return cuda_fail(err, err_len, e, "cudaMalloc");
    if ((e = cudaMemset(*dptr, 0, bytes)) != cudaSuccess) {
        cudaFree(*dptr);
        *dptr = nullptr;
        return cuda_fail(err, err_len, e, "cudaMemset");
    }
    return DM_OK;
}

extern "C" int dm_device_free(void *dptr, char *err, size_t err_len) {
    if (!dptr) return fail(err, err_len, DM_EINVAL, "dm_device_free: null pointer");
    cudaError_t e = cudaFree(dptr);
    if (e != cudaSuccess) return cuda_fail(err, err_len, e, "cudaFree");
    return DM_OK;
}

extern "C" int64_t dm_prefill_workspace_bytes(const dm_tensor *t, int64_t M) {
    if (!t || M < 1) return 0;
    return dm::prefill_workspace_bytes(t, M);
}

extern "C" int dm_prefill(const dm_tensor *t, const void *x, int64_t M, const void *bias, void *out,
                          int32_t out_dtype, void *work, int64_t work_bytes, void *stream, char *err,
                          size_t err_len) {
    if (!t || !x || !out || !work) return fail(err, err_len, DM_EINVAL, "dm_prefill: null pointer");
    if (M < 1) return fail(err, err_len, DM_EINVAL, "dm_prefill: M must be at least 1");
    if (out_dtype != DM_BF16 && out_dtype != DM_F32)
        return fail(err, err_len, DM_EINVAL, "dm_prefill: dtype must be DM_BF16 or DM_F32");
    DeviceGuard g(t->device);
    std::string msg;
    int rc = dm::launch_prefill_sip(t, reinterpret_cast<const uint16_t *>(x), M, reinterpret_cast<const uint16_t *>(bias),
                                    out, out_dtype == DM_F32, reinterpret_cast<uint8_t *>(work), work_bytes, stream, msg);
    if (rc) dm::set_error(err, err_len, msg);
    return rc;
}
