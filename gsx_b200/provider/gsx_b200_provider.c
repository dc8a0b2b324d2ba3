/*
 * GSX backend provider over the gsx-b200 C ABI: the B200 kernels dropped in behind GSX's own
 * backend/buffer/renderer/loss/optimizer vtables (gsx/src/gsx-impl.h:220-491), unchanged GSX
 * front-ends on top.
 *
 * It is the CUDA backend type of GSX (GSX_BACKEND_TYPE_CUDA, name "cuda"): it defines
 * gsx_cuda_backend_provider_bootstrap, the symbol that gsx_backend_registry_init calls when GSX is
 * compiled with GSX_HAS_CUDA=1 (gsx/src/gsx-backend.c:226), so a GSX build links this file plus
 * libgsx_b200.so in place of its gsx/src/gsx-cuda/ sources and no GSX source changes.
 *
 * Scope (the training hot path and what density control needs around it): device and pinned-host
 * buffers with the buffer operations the GSX core and front-ends issue on that path
 * (upload/download, set/get/memset/copy/fill, finiteness, row gather, clamp); the renderer (float32
 * RGB forward INFERENCE/TRAIN with borrowed or cloned train state, RGB backward, the density-control
 * statistics of the requests); L1/MSE/SSIM losses with MEAN/SUM gradient normalisation; Adam with its
 * structural ops (permute, gather, resize, reset); the default ADC.  Everything else returns
 * GSX_ERROR_NOT_SUPPORTED, as the reference CUDA backend does for what it lacks
 * (gsx-cuda/render.c:766-800, 1583-1592): unary/reduce tensor math, random fills, image conversion,
 * the async dataloader and the MCMC ADC.
 *
 * Build: compiled against a GSX source tree's headers (gsx/include and gsx/src for gsx-impl.h), see
 * gsx_b200/provider/Makefile.  All work runs on the backend's major stream (gsx-base.h:94-109).
 */
#include "gsx-impl.h"

#include "gsx_b200.h"

#include <cuda_runtime.h>
#include <float.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define B200_MAX_DEVICES 64

/* ------------------------------------------------------------------------------------------ */
/* errors */

static gsx_error b200_ok(void) { return gsx_make_error(GSX_ERROR_SUCCESS, NULL); }

static gsx_error b200_cuda_error(cudaError_t e, const char *what)
{
    if(e == cudaSuccess) return b200_ok();
    if(e == cudaErrorMemoryAllocation) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, what);
    return gsx_make_error(GSX_ERROR_UNKNOWN, what);
}

/* gsx-b200 return codes are gsx_error_code values; the message is static per call site */
static gsx_error b200_lib_error(int rc, const char *what)
{
    if(rc == GSX_B200_SUCCESS) return b200_ok();
    return gsx_make_error((gsx_error_code)rc, what);
}

#define B200_TRY(expr)                                      \
    do {                                                    \
        gsx_error e__ = (expr);                             \
        if(!gsx_error_is_success(e__)) return e__;          \
    } while(0)

/* ------------------------------------------------------------------------------------------ */
/* provider, devices, backend, buffer types, buffers */

typedef struct b200_device {
    struct gsx_backend_device base;
    int ordinal;
    char name[256];
} b200_device;

typedef struct b200_backend b200_backend;

typedef struct b200_buffer_type {
    struct gsx_backend_buffer_type base;
    gsx_backend_buffer_type_class type_class;
    const char *name;
    gsx_size_t alignment;
} b200_buffer_type;

struct b200_backend {
    struct gsx_backend base;
    int ordinal;
    cudaStream_t stream;
    gsx_backend_capabilities caps;
    b200_buffer_type device_type;
    b200_buffer_type pinned_type;
    uint32_t *finite_word; /* device word for check_finite_tensor */
};

typedef struct b200_buffer {
    struct gsx_backend_buffer base;
    void *ptr;
} b200_buffer;

static struct gsx_backend_provider b200_provider;
static b200_device b200_devices[B200_MAX_DEVICES];

static b200_backend *b200_backend_of(gsx_backend_t backend) { return (b200_backend *)backend; }
static b200_buffer_type *b200_type_of(gsx_backend_buffer_type_t t) { return (b200_buffer_type *)t; }
static b200_buffer *b200_buffer_of(gsx_backend_buffer_t b) { return (b200_buffer *)b; }
static b200_backend *b200_backend_of_buffer(gsx_backend_buffer_t b) { return b200_backend_of(b->buffer_type->backend); }

static bool b200_is_device(gsx_backend_buffer_t b)
{
    return b != NULL && b200_type_of(b->buffer_type)->type_class == GSX_BACKEND_BUFFER_TYPE_DEVICE;
}

static unsigned char *b200_view_ptr(const gsx_backend_tensor_view *view)
{
    return (unsigned char *)b200_buffer_of(view->buffer)->ptr + (size_t)view->offset_bytes;
}

/* device pointer of a GSX tensor that lives in one of this backend's device buffers, or NULL */
static float *b200_tensor_f32(gsx_tensor_t t)
{
    if(t == NULL || t->backing_buffer == NULL || !b200_is_device(t->backing_buffer)) return NULL;
    return (float *)((unsigned char *)b200_buffer_of(t->backing_buffer)->ptr + (size_t)t->offset_bytes);
}

static int32_t *b200_tensor_i32(gsx_tensor_t t) { return (int32_t *)b200_tensor_f32(t); }

static gsx_error b200_sync(b200_backend *be) { return b200_cuda_error(cudaStreamSynchronize(be->stream), "cudaStreamSynchronize failed"); }

/* buffer interface ------------------------------------------------------------------------ */

static gsx_error b200_buffer_free(gsx_backend_buffer_t buffer)
{
    b200_buffer *b = b200_buffer_of(buffer);
    b200_backend *be = b200_backend_of_buffer(buffer);
    cudaError_t e = cudaSetDevice(be->ordinal);
    if(e == cudaSuccess) e = cudaStreamSynchronize(be->stream);
    if(e == cudaSuccess && b->ptr != NULL)
        e = b200_is_device(buffer) ? cudaFree(b->ptr) : cudaFreeHost(b->ptr);
    if(e != cudaSuccess) return b200_cuda_error(e, "buffer free failed");
    if(be->base.live_buffer_count > 0) be->base.live_buffer_count -= 1;
    free(b);
    return b200_ok();
}

static gsx_error b200_buffer_get_info(gsx_backend_buffer_t buffer, gsx_backend_buffer_info *out)
{
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_info must be non-null");
    out->backend = buffer->buffer_type->backend;
    out->buffer_type = buffer->buffer_type;
    out->size_bytes = buffer->size_bytes;
    out->alignment_bytes = buffer->alignment_bytes;
    return b200_ok();
}

static gsx_error b200_buffer_native(gsx_backend_buffer_t buffer, void **out)
{
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_handle must be non-null");
    *out = b200_buffer_of(buffer)->ptr;
    return b200_ok();
}

/* host bytes <-> buffer bytes, stream ordered, complete on return */
static gsx_error b200_copy_host(gsx_backend_buffer_t buffer, size_t offset, void *host, const void *src_host, size_t n,
                                bool to_buffer)
{
    b200_backend *be = b200_backend_of_buffer(buffer);
    unsigned char *p = (unsigned char *)b200_buffer_of(buffer)->ptr + offset;
    if(n == 0) return b200_ok();
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    cudaError_t e = to_buffer ? cudaMemcpyAsync(p, src_host, n, cudaMemcpyDefault, be->stream)
                              : cudaMemcpyAsync(host, p, n, cudaMemcpyDefault, be->stream);
    if(e != cudaSuccess) return b200_cuda_error(e, "cudaMemcpyAsync failed");
    return b200_sync(be);
}

static gsx_error b200_buffer_upload(gsx_backend_buffer_t buffer, gsx_size_t dst_offset, const void *src, gsx_size_t n)
{
    if(dst_offset > buffer->size_bytes || n > buffer->size_bytes - dst_offset)
        return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "upload range exceeds the buffer");
    return b200_copy_host(buffer, (size_t)dst_offset, NULL, src, (size_t)n, true);
}

static gsx_error b200_buffer_download(gsx_backend_buffer_t buffer, gsx_size_t src_offset, void *dst, gsx_size_t n)
{
    if(src_offset > buffer->size_bytes || n > buffer->size_bytes - src_offset)
        return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "download range exceeds the buffer");
    return b200_copy_host(buffer, (size_t)src_offset, dst, NULL, (size_t)n, false);
}

static gsx_error b200_buffer_set_zero(gsx_backend_buffer_t buffer)
{
    b200_backend *be = b200_backend_of_buffer(buffer);
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    return b200_cuda_error(cudaMemsetAsync(b200_buffer_of(buffer)->ptr, 0, (size_t)buffer->size_bytes, be->stream),
                           "cudaMemsetAsync failed");
}

static gsx_error b200_buffer_memset_tensor(gsx_backend_buffer_t buffer, const gsx_backend_tensor_view *view, uint8_t value,
                                           gsx_size_t offset, gsx_size_t size)
{
    b200_backend *be = b200_backend_of_buffer(buffer);
    if(offset > view->size_bytes || size > view->size_bytes - offset)
        return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "memset range exceeds the tensor");
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    return b200_cuda_error(cudaMemsetAsync(b200_view_ptr(view) + offset, value, (size_t)size, be->stream), "cudaMemsetAsync failed");
}

static gsx_error b200_buffer_set_tensor(gsx_backend_buffer_t buffer, const gsx_backend_tensor_view *view, const void *src,
                                        gsx_size_t offset, gsx_size_t size)
{
    if(offset > view->size_bytes || size > view->size_bytes - offset)
        return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "set range exceeds the tensor");
    return b200_copy_host(buffer, (size_t)(view->offset_bytes + offset), NULL, src, (size_t)size, true);
}

static gsx_error b200_buffer_get_tensor(gsx_backend_buffer_t buffer, const gsx_backend_tensor_view *view, void *dst,
                                        gsx_size_t offset, gsx_size_t size)
{
    if(offset > view->size_bytes || size > view->size_bytes - offset)
        return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "get range exceeds the tensor");
    return b200_copy_host(buffer, (size_t)(view->offset_bytes + offset), dst, NULL, (size_t)size, false);
}

static gsx_error b200_buffer_copy_tensor(gsx_backend_buffer_t dst_buffer, const gsx_backend_tensor_view *src_view,
                                         const gsx_backend_tensor_view *dst_view)
{
    b200_backend *be = b200_backend_of_buffer(dst_buffer);
    if(src_view->size_bytes != dst_view->size_bytes) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "copy size mismatch");
    if(src_view->buffer->buffer_type->backend != dst_buffer->buffer_type->backend)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "copy across backends is not supported");
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    return b200_cuda_error(cudaMemcpyAsync(b200_view_ptr(dst_view), b200_view_ptr(src_view), (size_t)src_view->size_bytes,
                                           cudaMemcpyDefault, be->stream),
                           "cudaMemcpyAsync failed");
}

static gsx_error b200_buffer_fill_tensor(gsx_backend_buffer_t buffer, const gsx_backend_tensor_view *view, const void *value,
                                         gsx_size_t value_size)
{
    b200_backend *be = b200_backend_of_buffer(buffer);
    if(value == NULL || value_size == 0) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "fill value must be non-empty");
    if(!b200_is_device(buffer)) {
        /* pinned host memory: fill on the host after the stream's pending work */
        B200_TRY(b200_sync(be));
        for(gsx_size_t o = 0; o + value_size <= view->size_bytes; o += value_size) memcpy(b200_view_ptr(view) + o, value, value_size);
        return b200_ok();
    }
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    return b200_lib_error(gsx_b200_fill_pattern(b200_view_ptr(view), view->size_bytes, value, (uint32_t)value_size, be->stream),
                          "gsx_b200_fill_pattern failed");
}

static gsx_error b200_buffer_check_finite(gsx_backend_buffer_t buffer, const gsx_backend_tensor_view *view, bool *out)
{
    b200_backend *be = b200_backend_of_buffer(buffer);
    uint32_t bad = 0;
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_is_finite must be non-null");
    if(view->data_type != GSX_DATA_TYPE_F32) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "finiteness check supports float32 only");
    if(!b200_is_device(buffer)) {
        const float *x = (const float *)b200_view_ptr(view);
        B200_TRY(b200_sync(be));
        for(gsx_size_t i = 0; i < view->size_bytes / 4; ++i) bad += isfinite(x[i]) ? 0u : 1u;
        *out = bad == 0;
        return b200_ok();
    }
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    B200_TRY(b200_cuda_error(cudaMemsetAsync(be->finite_word, 0, sizeof(uint32_t), be->stream), "cudaMemsetAsync failed"));
    B200_TRY(b200_lib_error(gsx_b200_count_nonfinite_f32((const float *)b200_view_ptr(view), view->size_bytes / 4, be->finite_word,
                                                         be->stream),
                            "gsx_b200_count_nonfinite_f32 failed"));
    B200_TRY(b200_cuda_error(cudaMemcpyAsync(&bad, be->finite_word, sizeof(bad), cudaMemcpyDeviceToHost, be->stream), "D2H failed"));
    B200_TRY(b200_sync(be));
    *out = bad == 0;
    return b200_ok();
}

/* operations outside the path: GSX_ERROR_NOT_SUPPORTED */
#define B200_UNSUPPORTED(name) gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 backend does not implement " name)

static gsx_error b200_fill_rand(gsx_backend_buffer_t b, const gsx_backend_tensor_view *v, uint64_t s, uint64_t i)
{
    (void)b, (void)v, (void)s, (void)i;
    return B200_UNSUPPORTED("random fills");
}
static gsx_error b200_fill_randn(gsx_backend_buffer_t b, const gsx_backend_tensor_view *v, uint64_t s, uint64_t i, gsx_float_t g)
{
    (void)b, (void)v, (void)s, (void)i, (void)g;
    return B200_UNSUPPORTED("random fills");
}
static gsx_error b200_fill_randint(gsx_backend_buffer_t b, const gsx_backend_tensor_view *v, uint64_t s, uint64_t i, uint32_t n)
{
    (void)b, (void)v, (void)s, (void)i, (void)n;
    return B200_UNSUPPORTED("random fills");
}
static gsx_error b200_multinomial(gsx_backend_buffer_t b, const gsx_backend_tensor_view *o, const gsx_backend_tensor_view *c,
                                  uint64_t s, uint64_t i)
{
    (void)b, (void)o, (void)c, (void)s, (void)i;
    return B200_UNSUPPORTED("multinomial sampling");
}
/* rows of x gathered by an int32 index (gsx-impl.h:373-382; gsx-cuda/buffer.c:1120-1240): the
 * density-control path's gsx_gs_gather.  An out-of-range index fails with OUT_OF_RANGE. */
static gsx_error b200_gather(gsx_backend_buffer_t b, const gsx_backend_tensor_view *x, const gsx_backend_tensor_view *ix,
                             const gsx_backend_tensor_view *o, gsx_index_t xr, const gsx_index_t *xs, gsx_index_t orr,
                             const gsx_index_t *os)
{
    b200_backend *be = b200_backend_of_buffer(b);
    uint32_t bad = 0;
    gsx_size_t rows = 0, row_bytes = 0;
    if(x == NULL || ix == NULL || o == NULL || xs == NULL || os == NULL || xr < 1 || orr < 1)
        return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "gather views and shapes must be non-null");
    if(ix->data_type != GSX_DATA_TYPE_I32) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "gather index must be int32");
    rows = (gsx_size_t)os[0];
    if(rows == 0) return b200_ok();
    if(o->size_bytes % rows != 0) return gsx_make_error(GSX_ERROR_INVALID_STATE, "gather output view byte size must be row-aligned");
    row_bytes = o->size_bytes / rows;
    if((gsx_size_t)xs[0] * row_bytes != x->size_bytes)
        return gsx_make_error(GSX_ERROR_INVALID_STATE, "gather x view byte size is inconsistent with row metadata");
    if(rows * sizeof(int32_t) != ix->size_bytes)
        return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "index view byte size must match out leading dimension");
    if(row_bytes == 0) return b200_ok();
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    if(!b200_is_device(b) || !b200_is_device(x->buffer) || !b200_is_device(ix->buffer)) {
        const unsigned char *src = b200_view_ptr(x);
        const int32_t *idx = (const int32_t *)b200_view_ptr(ix);
        unsigned char *dst = b200_view_ptr(o);
        if(b200_is_device(b) || b200_is_device(x->buffer) || b200_is_device(ix->buffer))
            return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gather across device and host buffers is not supported");
        B200_TRY(b200_sync(be));
        for(gsx_size_t r = 0; r < rows; ++r) {
            if(idx[r] < 0 || (gsx_size_t)idx[r] >= (gsx_size_t)xs[0]) return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "gather index is out of range");
            memcpy(dst + r * row_bytes, src + (gsx_size_t)idx[r] * row_bytes, (size_t)row_bytes);
        }
        return b200_ok();
    }
    B200_TRY(b200_cuda_error(cudaMemsetAsync(be->finite_word, 0, sizeof(uint32_t), be->stream), "cudaMemsetAsync failed"));
    B200_TRY(b200_lib_error(gsx_b200_gather_rows(b200_view_ptr(x), (uint64_t)xs[0], row_bytes, (const int32_t *)b200_view_ptr(ix),
                                                 rows, b200_view_ptr(o), be->finite_word, be->stream),
                            "gsx_b200_gather_rows failed"));
    B200_TRY(b200_cuda_error(cudaMemcpyAsync(&bad, be->finite_word, sizeof(bad), cudaMemcpyDeviceToHost, be->stream), "D2H failed"));
    B200_TRY(b200_sync(be));
    if(bad != 0) return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "gather index is out of range");
    return b200_ok();
}
static gsx_error b200_unary(gsx_backend_buffer_t b, const gsx_backend_tensor_view *x, const gsx_backend_tensor_view *o,
                            gsx_index_t r, const gsx_index_t *s, gsx_impl_unary_op op)
{
    (void)b, (void)x, (void)o, (void)r, (void)s, (void)op;
    return B200_UNSUPPORTED("unary tensor ops");
}
static gsx_error b200_unary_inplace(gsx_backend_buffer_t b, const gsx_backend_tensor_view *v, gsx_impl_unary_op op)
{
    (void)b, (void)v, (void)op;
    return B200_UNSUPPORTED("unary tensor ops");
}
static gsx_error b200_unary_reduce(gsx_backend_buffer_t b, const gsx_backend_tensor_view *x, const gsx_backend_tensor_view *o,
                                   const gsx_backend_tensor_view *w, gsx_index_t xr, const gsx_index_t *xs, gsx_index_t orr,
                                   const gsx_index_t *os, gsx_index_t a, gsx_impl_unary_reduce_op op)
{
    (void)b, (void)x, (void)o, (void)w, (void)xr, (void)xs, (void)orr, (void)os, (void)a, (void)op;
    return B200_UNSUPPORTED("tensor reductions");
}
static gsx_error b200_binary_reduce(gsx_backend_buffer_t b, const gsx_backend_tensor_view *l, const gsx_backend_tensor_view *r,
                                    const gsx_backend_tensor_view *o, const gsx_backend_tensor_view *w, gsx_index_t lr,
                                    const gsx_index_t *ls, gsx_index_t rr, const gsx_index_t *rs, gsx_index_t orr,
                                    const gsx_index_t *os, gsx_index_t a, gsx_impl_binary_reduce_op op)
{
    (void)b, (void)l, (void)r, (void)o, (void)w, (void)lr, (void)ls, (void)rr, (void)rs, (void)orr, (void)os, (void)a, (void)op;
    return B200_UNSUPPORTED("tensor reductions");
}
/* in-place clamp (gsx-cuda/buffer.c:1985-2060): density control's opacity reset */
static gsx_error b200_clamp(gsx_backend_buffer_t b, const gsx_backend_tensor_view *v, const void *lo, const void *hi)
{
    b200_backend *be = b200_backend_of_buffer(b);
    gsx_size_t es = 0;
    if(v == NULL || lo == NULL || hi == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "clamp view and bounds must be non-null");
    if(v->data_type == GSX_DATA_TYPE_F32 || v->data_type == GSX_DATA_TYPE_I32) es = 4;
    else if(v->data_type == GSX_DATA_TYPE_U8) es = 1;
    else return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "clamp supports float32, int32 and uint8");
    if(v->size_bytes % es != 0) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "tensor view byte size is not aligned to element size");
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    if(!b200_is_device(b)) {
        unsigned char *p = b200_view_ptr(v);
        B200_TRY(b200_sync(be));
        for(gsx_size_t i = 0; i < v->size_bytes / es; ++i) {
            if(v->data_type == GSX_DATA_TYPE_F32) {
                float *x = (float *)p + i;
                if(*x < *(const float *)lo) *x = *(const float *)lo;
                else if(*x > *(const float *)hi) *x = *(const float *)hi;
            } else if(v->data_type == GSX_DATA_TYPE_I32) {
                int32_t *x = (int32_t *)p + i;
                if(*x < *(const int32_t *)lo) *x = *(const int32_t *)lo;
                else if(*x > *(const int32_t *)hi) *x = *(const int32_t *)hi;
            } else {
                uint8_t *x = p + i;
                if(*x < *(const uint8_t *)lo) *x = *(const uint8_t *)lo;
                else if(*x > *(const uint8_t *)hi) *x = *(const uint8_t *)hi;
            }
        }
        return b200_ok();
    }
    return b200_lib_error(gsx_b200_clamp_inplace(b200_view_ptr(v), (int)v->data_type, v->size_bytes / es, lo, hi, be->stream),
                          "gsx_b200_clamp_inplace failed");
}
static gsx_error b200_img_colorspace(gsx_backend_buffer_t b, const gsx_backend_tensor_view *s, gsx_storage_format f,
                                     gsx_index_t r, const gsx_index_t *sh, gsx_image_colorspace sc,
                                     const gsx_backend_tensor_view *d, gsx_image_colorspace dc)
{
    (void)b, (void)s, (void)f, (void)r, (void)sh, (void)sc, (void)d, (void)dc;
    return B200_UNSUPPORTED("image conversion");
}
static gsx_error b200_img_storage(gsx_backend_buffer_t b, const gsx_backend_tensor_view *s, gsx_index_t sr, const gsx_index_t *ss,
                                  gsx_storage_format sf, const gsx_backend_tensor_view *d, gsx_index_t dr, const gsx_index_t *ds,
                                  gsx_storage_format df)
{
    (void)b, (void)s, (void)sr, (void)ss, (void)sf, (void)d, (void)dr, (void)ds, (void)df;
    return B200_UNSUPPORTED("image conversion");
}
static gsx_error b200_img_dtype(gsx_backend_buffer_t b, const gsx_backend_tensor_view *s, gsx_storage_format f, gsx_index_t r,
                                const gsx_index_t *sh, const gsx_backend_tensor_view *d)
{
    (void)b, (void)s, (void)f, (void)r, (void)sh, (void)d;
    return B200_UNSUPPORTED("image conversion");
}

static const gsx_backend_buffer_i b200_buffer_iface = {
    b200_buffer_free,        b200_buffer_get_info,     b200_buffer_native,       b200_buffer_upload,
    b200_buffer_download,    b200_buffer_set_zero,     b200_buffer_memset_tensor, b200_buffer_set_tensor,
    b200_buffer_get_tensor,  b200_buffer_copy_tensor,  b200_buffer_fill_tensor,  b200_fill_rand,
    b200_fill_randn,         b200_fill_randint,        b200_multinomial,         b200_buffer_check_finite,
    b200_gather,             b200_unary,               b200_unary_inplace,       b200_unary_reduce,
    b200_binary_reduce,      b200_clamp,               b200_img_colorspace,      b200_img_storage,
    b200_img_dtype,
};

/* buffer-type interface ------------------------------------------------------------------- */

static gsx_error b200_type_get_info(gsx_backend_buffer_type_t type, gsx_backend_buffer_type_info *out)
{
    b200_buffer_type *t = b200_type_of(type);
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_info must be non-null");
    out->backend = t->base.backend;
    out->type = t->type_class;
    out->name = t->name;
    out->alignment_bytes = t->alignment;
    out->max_allocation_size_bytes = 0;
    return b200_ok();
}

static gsx_error b200_type_alloc_size(gsx_backend_buffer_type_t type, gsx_size_t requested, gsx_size_t *out)
{
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_alloc_size_bytes must be non-null");
    if(gsx_round_up_overflows(requested, b200_type_of(type)->alignment, out))
        return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "allocation size overflows");
    return b200_ok();
}

static gsx_error b200_type_init_buffer(gsx_backend_buffer_type_t type, const gsx_backend_buffer_desc *desc, gsx_backend_buffer_t *out)
{
    b200_buffer_type *t = b200_type_of(type);
    b200_backend *be = b200_backend_of(t->base.backend);
    gsx_size_t align = desc->alignment_bytes ? desc->alignment_bytes : t->alignment;
    gsx_size_t bytes = 0;
    b200_buffer *b = NULL;
    cudaError_t e = cudaSuccess;
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_buffer must be non-null");
    *out = NULL;
    if(desc->size_bytes == 0) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "buffer size must be non-zero");
    if(!gsx_is_power_of_two(align)) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "alignment must be a power of two");
    /* cudaMalloc / cudaMallocHost return 256-byte aligned memory */
    if(align > 256) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "alignments above 256 bytes are not supported");
    if(gsx_round_up_overflows(desc->size_bytes, align, &bytes)) return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "buffer size overflows");
    b = (b200_buffer *)calloc(1, sizeof(*b));
    if(b == NULL) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate the buffer record");
    e = cudaSetDevice(be->ordinal);
    if(e == cudaSuccess) e = t->type_class == GSX_BACKEND_BUFFER_TYPE_DEVICE ? cudaMalloc(&b->ptr, (size_t)bytes)
                                                                              : cudaMallocHost(&b->ptr, (size_t)bytes);
    if(e != cudaSuccess) {
        free(b);
        return b200_cuda_error(e, "buffer allocation failed");
    }
    b->base.iface = &b200_buffer_iface;
    b->base.buffer_type = type;
    b->base.size_bytes = desc->size_bytes;
    b->base.alignment_bytes = align;
    be->base.live_buffer_count += 1;
    *out = &b->base;
    return b200_ok();
}

static const gsx_backend_buffer_type_i b200_type_iface = { b200_type_get_info, b200_type_alloc_size, b200_type_init_buffer };

/* ------------------------------------------------------------------------------------------ */
/* renderer */

typedef struct b200_renderer {
    struct gsx_renderer base;
} b200_renderer;

typedef struct b200_render_context {
    struct gsx_render_context base;
    gsx_b200_context *ctx;
    float *clone;          /* TRAIN state cloned from the inputs when the caller does not lend it */
    size_t clone_bytes;
    bool has_train;
    bool train_cloned;
} b200_render_context;

static gsx_error b200_renderer_destroy(gsx_renderer_t renderer)
{
    if(renderer->live_context_count != 0) return gsx_make_error(GSX_ERROR_INVALID_STATE, "renderer has live contexts");
    gsx_renderer_base_deinit(renderer);
    free(renderer);
    return b200_ok();
}

static gsx_error b200_render_context_destroy(gsx_render_context_t context)
{
    b200_render_context *c = (b200_render_context *)context;
    b200_backend *be = b200_backend_of(context->renderer->backend);
    cudaSetDevice(be->ordinal);
    cudaStreamSynchronize(be->stream);
    if(c->ctx) gsx_b200_context_destroy(c->ctx);
    if(c->clone) cudaFree(c->clone);
    gsx_render_context_base_deinit(context);
    free(c);
    return b200_ok();
}

static const gsx_render_context_i b200_render_context_iface = { b200_render_context_destroy };

static gsx_error b200_renderer_create_context(gsx_renderer_t renderer, gsx_render_context_t *out)
{
    b200_backend *be = b200_backend_of(renderer->backend);
    b200_render_context *c = NULL;
    int rc = 0;
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_context must be non-null");
    *out = NULL;
    c = (b200_render_context *)calloc(1, sizeof(*c));
    if(c == NULL) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate the render context");
    rc = gsx_b200_context_create(be->ordinal, &c->ctx);
    if(rc != 0) {
        free(c);
        return b200_lib_error(rc, "gsx_b200_context_create failed");
    }
    gsx_error e = gsx_render_context_base_init(&c->base, &b200_render_context_iface, renderer);
    if(!gsx_error_is_success(e)) {
        gsx_b200_context_destroy(c->ctx);
        free(c);
        return e;
    }
    *out = &c->base;
    return b200_ok();
}

/* the request's Gaussian fields as device pointers; sh1..sh3 only up to sh_degree */
static gsx_error b200_gaussians_of(const gsx_render_forward_request *r, gsx_b200_gaussians *g)
{
    memset(g, 0, sizeof(*g));
    g->count = r->gs_mean3d ? (int64_t)r->gs_mean3d->shape[0] : 0;
    g->mean3d = b200_tensor_f32(r->gs_mean3d);
    g->rotation = b200_tensor_f32(r->gs_rotation);
    g->logscale = b200_tensor_f32(r->gs_logscale);
    g->opacity = b200_tensor_f32(r->gs_opacity);
    g->sh0 = b200_tensor_f32(r->gs_sh0);
    if(r->sh_degree >= 1) g->sh1 = b200_tensor_f32(r->gs_sh1);
    if(r->sh_degree >= 2) g->sh2 = b200_tensor_f32(r->gs_sh2);
    if(r->sh_degree >= 3) g->sh3 = b200_tensor_f32(r->gs_sh3);
    if(g->count > 0 && (g->mean3d == NULL || g->rotation == NULL || g->logscale == NULL || g->opacity == NULL || g->sh0 == NULL))
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer requires device-backed Gaussian tensors");
    if((r->sh_degree >= 1 && g->sh1 == NULL) || (r->sh_degree >= 2 && g->sh2 == NULL) || (r->sh_degree >= 3 && g->sh3 == NULL))
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer requires device-backed SH tensors up to sh_degree");
    return b200_ok();
}

/* TRAIN without borrowing: retain a private copy of the Gaussian fields (the caller may change
 * its tensors before backward), as the reference's cloned train state (gsx-cuda/render.c:481-560) */
static gsx_error b200_clone_gaussians(b200_render_context *c, b200_backend *be, gsx_b200_gaussians *g, int sh_degree)
{
    static const int cols[8] = { 3, 4, 3, 1, 3, 9, 15, 21 };
    const float *src[8] = { g->mean3d, g->rotation, g->logscale, g->opacity, g->sh0, g->sh1, g->sh2, g->sh3 };
    const float **dst[8] = { &g->mean3d, &g->rotation, &g->logscale, &g->opacity, &g->sh0, &g->sh1, &g->sh2, &g->sh3 };
    const int nf = 5 + sh_degree;
    size_t off[8], total = 0;
    for(int f = 0; f < nf; ++f) {
        off[f] = total;
        total += ((size_t)g->count * (size_t)cols[f] * sizeof(float) + 255u) & ~(size_t)255u;
    }
    if(total > c->clone_bytes) {
        if(c->clone) cudaFree(c->clone);
        c->clone = NULL;
        c->clone_bytes = 0;
        B200_TRY(b200_cuda_error(cudaMalloc((void **)&c->clone, total), "clone allocation failed"));
        c->clone_bytes = total;
    }
    for(int f = 0; f < nf; ++f) {
        float *d = (float *)((unsigned char *)c->clone + off[f]);
        B200_TRY(b200_cuda_error(cudaMemcpyAsync(d, src[f], (size_t)g->count * (size_t)cols[f] * sizeof(float),
                                                 cudaMemcpyDeviceToDevice, be->stream),
                                 "clone copy failed"));
        *dst[f] = d;
    }
    return b200_ok();
}

static gsx_error b200_renderer_render(gsx_renderer_t renderer, gsx_render_context_t context, const gsx_render_forward_request *r)
{
    b200_render_context *c = (b200_render_context *)context;
    b200_backend *be = b200_backend_of(renderer->backend);
    gsx_b200_gaussians g;
    gsx_b200_camera cam;
    float *out = NULL;
    int rc = 0;
    /* what the reference CUDA backend also rejects (gsx-cuda/render.c:766-784) */
    if(r->precision != GSX_RENDER_PRECISION_FLOAT32)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer supports float32 precision only");
    if(r->forward_type == GSX_RENDER_FORWARD_TYPE_METRIC || r->metric_map != NULL || r->gs_metric_accumulator != NULL)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer does not implement metric mode");
    if(r->gs_cov3d != NULL) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer does not implement gs_cov3d input");
    if(r->out_invdepth != NULL || r->out_alpha != NULL)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer does not implement inverse-depth or alpha outputs");
    out = b200_tensor_f32(r->out_rgb);
    if(out == NULL) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer requires a device-backed out_rgb");
    B200_TRY(b200_gaussians_of(r, &g));
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    c->has_train = false;
    c->train_cloned = false;
    if(r->forward_type == GSX_RENDER_FORWARD_TYPE_TRAIN && !r->borrow_train_state && g.count > 0) {
        B200_TRY(b200_clone_gaussians(c, be, &g, (int)r->sh_degree));
        c->train_cloned = true;
    }
    memset(&cam, 0, sizeof(cam));
    cam.width = (int32_t)renderer->info.width;
    cam.height = (int32_t)renderer->info.height;
    cam.fx = r->intrinsics->fx;
    cam.fy = r->intrinsics->fy;
    cam.cx = r->intrinsics->cx;
    cam.cy = r->intrinsics->cy;
    cam.rot_xyzw[0] = r->pose->rot.x;
    cam.rot_xyzw[1] = r->pose->rot.y;
    cam.rot_xyzw[2] = r->pose->rot.z;
    cam.rot_xyzw[3] = r->pose->rot.w;
    cam.transl[0] = r->pose->transl.x;
    cam.transl[1] = r->pose->transl.y;
    cam.transl[2] = r->pose->transl.z;
    cam.near_plane = r->near_plane;
    cam.far_plane = r->far_plane;
    {
        const float bg[3] = { r->background_color.x, r->background_color.y, r->background_color.z };
        const int ft = r->forward_type == GSX_RENDER_FORWARD_TYPE_TRAIN ? GSX_B200_FORWARD_TRAIN : GSX_B200_FORWARD_INFERENCE;
        /* density-control statistics of a TRAIN forward (gsx-render.h:123-124) */
        rc = gsx_b200_render_bind_aux(c->ctx, b200_tensor_f32(r->gs_visible_counter), b200_tensor_f32(r->gs_max_screen_radius),
                                      NULL, NULL);
        /* borrowed TRAIN state: the backward re-renders if the caller changed the Gaussians in between
         * (gsx-cuda/render.c:662-756); cloned state: the copies above are what the backward reads */
        if(rc == 0)
            rc = gsx_b200_context_set_train_state(c->ctx, ft == GSX_B200_FORWARD_TRAIN && r->borrow_train_state
                                                              ? GSX_B200_TRAIN_STATE_BORROWED
                                                              : GSX_B200_TRAIN_STATE_RETAINED);
        if(rc == 0) rc = gsx_b200_render_forward(c->ctx, &g, (int)r->sh_degree, &cam, bg, ft, out, be->stream);
    }
    if(rc != 0) return b200_lib_error(rc, "gsx_b200_render_forward failed");
    c->has_train = r->forward_type == GSX_RENDER_FORWARD_TYPE_TRAIN;
    return b200_ok();
}

static gsx_error b200_renderer_backward(gsx_renderer_t renderer, gsx_render_context_t context, const gsx_render_backward_request *r)
{
    b200_render_context *c = (b200_render_context *)context;
    b200_backend *be = b200_backend_of(renderer->backend);
    gsx_b200_gaussian_grads gr;
    const float *grad_rgb = NULL;
    if(r->grad_invdepth != NULL || r->grad_alpha != NULL || r->grad_gs_cov3d != NULL)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer implements the RGB backward only");
    if(!c->has_train) return gsx_make_error(GSX_ERROR_INVALID_STATE, "backward requires a retained TRAIN forward on this context");
    grad_rgb = b200_tensor_f32(r->grad_rgb);
    memset(&gr, 0, sizeof(gr));
    gr.mean3d = b200_tensor_f32(r->grad_gs_mean3d);
    gr.rotation = b200_tensor_f32(r->grad_gs_rotation);
    gr.logscale = b200_tensor_f32(r->grad_gs_logscale);
    gr.opacity = b200_tensor_f32(r->grad_gs_opacity);
    gr.sh0 = b200_tensor_f32(r->grad_gs_sh0);
    gr.sh1 = b200_tensor_f32(r->grad_gs_sh1);
    gr.sh2 = b200_tensor_f32(r->grad_gs_sh2);
    gr.sh3 = b200_tensor_f32(r->grad_gs_sh3);
    if(grad_rgb == NULL || gr.mean3d == NULL || gr.rotation == NULL || gr.logscale == NULL || gr.opacity == NULL || gr.sh0 == NULL)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer requires device-backed gradient tensors");
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    /* density-control statistics of the backward (gsx-render.h:143-144) */
    B200_TRY(b200_lib_error(gsx_b200_render_bind_aux(c->ctx, NULL, NULL, b200_tensor_f32(r->gs_grad_acc),
                                                     b200_tensor_f32(r->gs_absgrad_acc)),
                            "gsx_b200_render_bind_aux failed"));
    return b200_lib_error(gsx_b200_render_backward(c->ctx, grad_rgb, &gr, be->stream), "gsx_b200_render_backward failed");
}

static const gsx_renderer_i b200_renderer_iface = { b200_renderer_destroy, b200_renderer_create_context, b200_renderer_render,
                                                    b200_renderer_backward };

static gsx_error b200_create_renderer(gsx_backend_t backend, const gsx_renderer_desc *desc, gsx_renderer_t *out)
{
    b200_renderer *rd = NULL;
    gsx_renderer_capabilities caps;
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_renderer must be non-null");
    *out = NULL;
    /* the reference CUDA renderer's capability set (gsx-cuda/render.c:1583-1607) */
    if(desc->output_data_type != GSX_DATA_TYPE_F32)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer supports float32 outputs only");
    if(desc->enable_alpha_output || desc->enable_invdepth_output)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer does not implement alpha or inverse-depth outputs");
    if((desc->feature_flags & GSX_RENDERER_FEATURE_ANTIALIASING) != 0)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 renderer does not implement anti-aliasing");
    rd = (b200_renderer *)calloc(1, sizeof(*rd));
    if(rd == NULL) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate the renderer");
    memset(&caps, 0, sizeof(caps));
    caps.supported_precisions = GSX_RENDER_PRECISION_FLAG_FLOAT32;
    gsx_error e = gsx_renderer_base_init(&rd->base, &b200_renderer_iface, backend, desc, &caps);
    if(!gsx_error_is_success(e)) {
        free(rd);
        return e;
    }
    *out = &rd->base;
    return b200_ok();
}

/* ------------------------------------------------------------------------------------------ */
/* losses */

typedef struct b200_loss_context {
    struct gsx_loss_context base;
} b200_loss_context;

static gsx_error b200_loss_destroy(gsx_loss_t loss)
{
    if(loss->live_context_count != 0) return gsx_make_error(GSX_ERROR_INVALID_STATE, "loss has live contexts");
    gsx_loss_base_deinit(loss);
    free(loss);
    return b200_ok();
}

static gsx_error b200_loss_context_destroy(gsx_loss_context_t context)
{
    gsx_loss_context_base_deinit(context);
    free(context);
    return b200_ok();
}

static const gsx_loss_context_i b200_loss_context_iface = { b200_loss_context_destroy };

static gsx_error b200_loss_create_context(gsx_loss_t loss, gsx_loss_context_t *out)
{
    b200_loss_context *c = NULL;
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_context must be non-null");
    c = (b200_loss_context *)calloc(1, sizeof(*c));
    if(c == NULL) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate the loss context");
    gsx_error e = gsx_loss_context_base_init(&c->base, &b200_loss_context_iface, loss);
    if(!gsx_error_is_success(e)) {
        free(c);
        return e;
    }
    *out = &c->base;
    return b200_ok();
}

/* [.., C, H, W] f32 CHW image planes: planes = product of the leading dimensions (the outer/channel
 * split of gsx-tensor-helpers.h:188-235 only matters through that product) */
static gsx_error b200_planes(gsx_tensor_t t, int64_t *planes, int32_t *h, int32_t *w)
{
    if(t->data_type != GSX_DATA_TYPE_F32) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 losses support float32 only");
    if(t->storage_format != GSX_STORAGE_FORMAT_CHW) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 SSIM supports CHW images only");
    if(t->rank < 3) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "SSIM needs a [C,H,W] or [B,C,H,W] tensor");
    *planes = 1;
    for(gsx_index_t d = 0; d + 2 < t->rank; ++d) *planes *= (int64_t)t->shape[d];
    *h = (int32_t)t->shape[t->rank - 2];
    *w = (int32_t)t->shape[t->rank - 1];
    return b200_ok();
}

static gsx_error b200_loss_forward(gsx_loss_t loss, gsx_loss_context_t context, const gsx_loss_forward_request *r)
{
    b200_backend *be = b200_backend_of(loss->backend);
    const float *p = b200_tensor_f32(r->prediction), *t = b200_tensor_f32(r->target);
    float *lm = b200_tensor_f32(r->loss_map_accumulator);
    (void)context;
    if(p == NULL || t == NULL || lm == NULL) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 losses require device tensors");
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    if(loss->algorithm == GSX_LOSS_ALGORITHM_SSIM) {
        int64_t planes = 0;
        int32_t h = 0, w = 0;
        B200_TRY(b200_planes(r->prediction, &planes, &h, &w));
        return b200_lib_error(gsx_b200_loss_l1_ssim(1, p, t, lm, NULL, NULL, planes, h, w, 0.0f, r->scale, 0.0f, 0.0f, be->stream),
                              "gsx_b200_loss_l1_ssim failed");
    }
    return b200_lib_error(gsx_b200_loss_pointwise(loss->algorithm == GSX_LOSS_ALGORITHM_L1 ? 0 : 2, p, t, lm,
                                                  r->prediction->size_bytes / sizeof(float), r->scale, be->stream),
                          "gsx_b200_loss_pointwise failed");
}

static gsx_error b200_loss_backward(gsx_loss_t loss, gsx_loss_context_t context, const gsx_loss_backward_request *r)
{
    b200_backend *be = b200_backend_of(loss->backend);
    const float *p = b200_tensor_f32(context->retained_prediction), *t = b200_tensor_f32(context->retained_target);
    float *g = b200_tensor_f32(r->grad_prediction_accumulator);
    const gsx_size_t n = context->retained_prediction->size_bytes / sizeof(float);
    /* gradient normalisation of gsx-tensor-helpers.h:236-244 (MEAN: scale / element count) */
    const float gs = loss->grad_normalization == GSX_LOSS_GRAD_NORMALIZATION_TYPE_MEAN ? r->scale / (float)n : r->scale;
    if(p == NULL || t == NULL || g == NULL) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 losses require device tensors");
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    if(loss->algorithm == GSX_LOSS_ALGORITHM_SSIM) {
        int64_t planes = 0;
        int32_t h = 0, w = 0;
        B200_TRY(b200_planes(context->retained_prediction, &planes, &h, &w));
        return b200_lib_error(gsx_b200_loss_l1_ssim(2, p, t, NULL, g, NULL, planes, h, w, 0.0f, 0.0f, 0.0f, gs, be->stream),
                              "gsx_b200_loss_l1_ssim failed");
    }
    return b200_lib_error(gsx_b200_loss_pointwise(loss->algorithm == GSX_LOSS_ALGORITHM_L1 ? 1 : 3, p, t, g, n, gs, be->stream),
                          "gsx_b200_loss_pointwise failed");
}

static const gsx_loss_i b200_loss_iface = { b200_loss_destroy, b200_loss_create_context, b200_loss_forward, b200_loss_backward };

static gsx_error b200_create_loss(gsx_backend_t backend, const gsx_loss_desc *desc, gsx_loss_t *out)
{
    struct gsx_loss *l = NULL;
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_loss must be non-null");
    *out = NULL;
    l = (struct gsx_loss *)calloc(1, sizeof(*l));
    if(l == NULL) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate the loss");
    gsx_error e = gsx_loss_base_init(l, &b200_loss_iface, backend, desc);
    if(!gsx_error_is_success(e)) {
        free(l);
        return e;
    }
    *out = l;
    return b200_ok();
}

/* ------------------------------------------------------------------------------------------ */
/* Adam */

typedef struct b200_optim {
    struct gsx_optim base;
    float **m1, **m2;     /* per group, device, parameter-sized */
    uint64_t *counts;     /* elements per group */
    uint64_t *steps;      /* Adam step counter per group (bias correction) */
    uint64_t *rows;       /* leading extent (Gaussians) the moments currently hold, per group */
} b200_optim;

static gsx_error b200_optim_free_state(b200_optim *o)
{
    for(gsx_index_t i = 0; i < o->base.param_group_count; ++i) {
        if(o->m1 && o->m1[i]) cudaFree(o->m1[i]);
        if(o->m2 && o->m2[i]) cudaFree(o->m2[i]);
    }
    free(o->m1);
    free(o->m2);
    free(o->counts);
    free(o->steps);
    free(o->rows);
    return b200_ok();
}

static gsx_error b200_optim_destroy(gsx_optim_t optim)
{
    b200_optim *o = (b200_optim *)optim;
    b200_backend *be = b200_backend_of(optim->backend);
    cudaSetDevice(be->ordinal);
    cudaStreamSynchronize(be->stream);
    b200_optim_free_state(o);
    gsx_optim_base_deinit(optim);
    free(o);
    return b200_ok();
}

static gsx_error b200_optim_step_selected(gsx_optim_t optim, const bool *selected)
{
    b200_optim *o = (b200_optim *)optim;
    b200_backend *be = b200_backend_of(optim->backend);
    gsx_b200_adam_group groups[16];
    int n = 0;
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    for(gsx_index_t i = 0; i < optim->param_group_count; ++i) {
        const gsx_optim_param_group_desc *pg = &optim->param_groups[i];
        if(selected != NULL && !selected[i]) continue;
        if(o->steps[i] == UINT64_MAX) return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "optimizer Adam step counter overflowed");
        float *param = b200_tensor_f32(pg->parameter);
        const float *grad = b200_tensor_f32(pg->gradient);
        if(param == NULL || grad == NULL) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 Adam requires device tensors");
        o->steps[i] += 1;
        /* bias corrections in double on the host, as gsx-cuda/optim.c:776-778 */
        groups[n].parameter = param;
        groups[n].gradient = grad;
        groups[n].first_moment = o->m1[i];
        groups[n].second_moment = o->m2[i];
        groups[n].count = o->counts[i];
        groups[n].learning_rate = optim->learning_rates[i];
        groups[n].beta1 = pg->beta1;
        groups[n].beta2 = pg->beta2;
        groups[n].epsilon = pg->epsilon;
        groups[n].weight_decay = pg->weight_decay;
        groups[n].max_grad = pg->max_grad;
        groups[n].inv_bias_correction1 = 1.0 / (1.0 - pow((double)pg->beta1, (double)o->steps[i]));
        groups[n].inv_bias_correction2 = 1.0 / (1.0 - pow((double)pg->beta2, (double)o->steps[i]));
        n += 1;
        if(n == 16) {
            B200_TRY(b200_lib_error(gsx_b200_adam_step(groups, n, be->stream), "gsx_b200_adam_step failed"));
            n = 0;
        }
    }
    if(n > 0) B200_TRY(b200_lib_error(gsx_b200_adam_step(groups, n, be->stream), "gsx_b200_adam_step failed"));
    return b200_ok();
}

static gsx_error b200_optim_reset_by_index(gsx_optim_t optim, gsx_index_t index)
{
    b200_optim *o = (b200_optim *)optim;
    b200_backend *be = b200_backend_of(optim->backend);
    if(index < 0 || index >= optim->param_group_count) return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "param-group index out of range");
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    B200_TRY(b200_cuda_error(cudaMemsetAsync(o->m1[index], 0, o->counts[index] * sizeof(float), be->stream), "memset failed"));
    B200_TRY(b200_cuda_error(cudaMemsetAsync(o->m2[index], 0, o->counts[index] * sizeof(float), be->stream), "memset failed"));
    o->steps[index] = 0;
    return b200_ok();
}

static gsx_error b200_optim_reset_all(gsx_optim_t optim)
{
    for(gsx_index_t i = 0; i < optim->param_group_count; ++i) B200_TRY(b200_optim_reset_by_index(optim, i));
    return b200_ok();
}

/* ---- structural ops of density control (gsx-cuda/optim.c:846-1195): the moments follow the
 * Gaussians when the set is permuted, gathered (grown / pruned) or resized.  New moment buffers are
 * filled first and swapped in only when everything succeeded, so a failing call leaves the state. */

/* leading extent of a parameter tensor (its Gaussian count) */
static gsx_size_t b200_rows_of(gsx_tensor_t t) { return t != NULL && t->rank >= 1 ? (gsx_size_t)t->shape[0] : 0; }

/* the common old / new Gaussian counts of all groups, with matching row widths */
static gsx_error b200_optim_transition(b200_optim *o, gsx_size_t *old_rows, gsx_size_t *new_rows, const char *what)
{
    for(gsx_index_t i = 0; i < o->base.param_group_count; ++i) {
        const gsx_tensor_t p = o->base.param_groups[i].parameter;
        const gsx_size_t orow = o->rows[i], nrow = b200_rows_of(p);
        const gsx_size_t elems = p->size_bytes / sizeof(float);
        if(orow == 0 || nrow == 0 || o->counts[i] % orow != 0 || elems % nrow != 0 || o->counts[i] / orow != elems / nrow)
            return gsx_make_error(GSX_ERROR_INVALID_STATE, "optimizer state and parameter row layouts do not match");
        if(i == 0) {
            *old_rows = orow;
            *new_rows = nrow;
        } else if(orow != *old_rows || nrow != *new_rows) {
            return gsx_make_error(GSX_ERROR_INVALID_STATE, what);
        }
    }
    return b200_ok();
}

/* rank-1 int32 device tensor of `count` entries, downloaded for validation */
static gsx_error b200_optim_indices(b200_optim *o, gsx_tensor_t t, gsx_size_t count, int32_t **out, const char *msg)
{
    b200_backend *be = b200_backend_of(o->base.backend);
    *out = NULL;
    if(t->rank != 1 || t->data_type != GSX_DATA_TYPE_I32 || (gsx_size_t)t->shape[0] != count || b200_tensor_i32(t) == NULL)
        return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, msg);
    *out = (int32_t *)malloc((size_t)(count ? count : 1) * sizeof(int32_t));
    if(*out == NULL) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate optimizer index validation storage");
    B200_TRY(b200_cuda_error(cudaMemcpyAsync(*out, b200_tensor_i32(t), (size_t)count * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                             be->stream),
                             "index download failed"));
    return b200_sync(be);
}

/* new moments: rows gathered by `index` (device, new_rows entries), or (index == NULL) the first
 * min(old, new) rows copied and the rest zero */
static gsx_error b200_optim_rebuild(b200_optim *o, gsx_size_t old_rows, gsx_size_t new_rows, const int32_t *index)
{
    b200_backend *be = b200_backend_of(o->base.backend);
    const gsx_index_t ng = o->base.param_group_count;
    float **n1 = (float **)calloc((size_t)ng, sizeof(float *)), **n2 = (float **)calloc((size_t)ng, sizeof(float *));
    gsx_error err = b200_ok();
    if(n1 == NULL || n2 == NULL) {
        free(n1);
        free(n2);
        return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate optimizer state records");
    }
    for(gsx_index_t i = 0; i < ng && gsx_error_is_success(err); ++i) {
        const gsx_size_t width = o->counts[i] / old_rows, bytes = new_rows * width * sizeof(float);
        float *src[2] = { o->m1[i], o->m2[i] };
        float **dst[2] = { &n1[i], &n2[i] };
        for(int m = 0; m < 2 && gsx_error_is_success(err); ++m) {
            err = b200_cuda_error(cudaMalloc((void **)dst[m], (size_t)(bytes ? bytes : sizeof(float))), "optimizer state allocation failed");
            if(!gsx_error_is_success(err)) break;
            if(index != NULL) {
                err = b200_lib_error(gsx_b200_gather_rows(src[m], old_rows, width * sizeof(float), index, new_rows, *dst[m], NULL,
                                                          be->stream),
                                     "gsx_b200_gather_rows failed");
            } else {
                const gsx_size_t keep = (old_rows < new_rows ? old_rows : new_rows) * width * sizeof(float);
                err = b200_cuda_error(cudaMemsetAsync(*dst[m], 0, (size_t)bytes, be->stream), "cudaMemsetAsync failed");
                if(gsx_error_is_success(err) && keep)
                    err = b200_cuda_error(cudaMemcpyAsync(*dst[m], src[m], (size_t)keep, cudaMemcpyDeviceToDevice, be->stream),
                                          "cudaMemcpyAsync failed");
            }
        }
    }
    if(gsx_error_is_success(err)) err = b200_sync(be);
    for(gsx_index_t i = 0; i < ng; ++i) {
        if(gsx_error_is_success(err)) {
            cudaFree(o->m1[i]);
            cudaFree(o->m2[i]);
            o->m1[i] = n1[i];
            o->m2[i] = n2[i];
            o->counts[i] = new_rows * (o->counts[i] / old_rows);
            o->rows[i] = new_rows;
        } else {
            if(n1[i]) cudaFree(n1[i]);
            if(n2[i]) cudaFree(n2[i]);
        }
    }
    free(n1);
    free(n2);
    return err;
}

static gsx_error b200_optim_permute(gsx_optim_t optim, gsx_tensor_t permutation)
{
    b200_optim *o = (b200_optim *)optim;
    b200_backend *be = b200_backend_of(optim->backend);
    gsx_size_t old_rows = 0, new_rows = 0;
    int32_t *idx = NULL;
    bool *seen = NULL;
    gsx_error err;
    if(optim->param_group_count == 0) return b200_ok();
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    B200_TRY(b200_optim_transition(o, &old_rows, &new_rows, "optimizer param groups must share the same leading extent for permutation"));
    if(old_rows != new_rows) return gsx_make_error(GSX_ERROR_INVALID_STATE, "optimizer permutation requires an unchanged leading extent");
    err = b200_optim_indices(o, permutation, old_rows, &idx, "optimizer permutation tensor must be rank-1 int32");
    if(gsx_error_is_success(err)) {
        seen = (bool *)calloc((size_t)old_rows, sizeof(bool));
        if(seen == NULL) err = gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate optimizer permutation validation storage");
    }
    for(gsx_size_t r = 0; r < old_rows && gsx_error_is_success(err); ++r) {
        if(idx[r] < 0) err = gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "optimizer permutation entries must be non-negative");
        else if((gsx_size_t)idx[r] >= old_rows) err = gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "optimizer permutation entries must be in range");
        else if(seen[idx[r]]) err = gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "optimizer permutation entries must be unique");
        else seen[idx[r]] = true;
    }
    free(seen);
    free(idx);
    if(!gsx_error_is_success(err)) return err;
    return b200_optim_rebuild(o, old_rows, new_rows, b200_tensor_i32(permutation));
}

static gsx_error b200_optim_gather(gsx_optim_t optim, gsx_tensor_t indices)
{
    b200_optim *o = (b200_optim *)optim;
    b200_backend *be = b200_backend_of(optim->backend);
    gsx_size_t old_rows = 0, new_rows = 0;
    int32_t *idx = NULL;
    gsx_error err;
    if(optim->param_group_count == 0) return b200_ok();
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    B200_TRY(b200_optim_transition(o, &old_rows, &new_rows, "optimizer param groups must share the same leading extents for gather"));
    err = b200_optim_indices(o, indices, new_rows, &idx, "optimizer indices tensor must be rank-1 int32");
    for(gsx_size_t r = 0; r < new_rows && gsx_error_is_success(err); ++r)
        if(idx[r] < 0 || (gsx_size_t)idx[r] >= old_rows) err = gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "optimizer gather indices must be in range");
    free(idx);
    if(!gsx_error_is_success(err)) return err;
    return b200_optim_rebuild(o, old_rows, new_rows, b200_tensor_i32(indices));
}

static gsx_error b200_optim_resize(gsx_optim_t optim, gsx_size_t count)
{
    b200_optim *o = (b200_optim *)optim;
    b200_backend *be = b200_backend_of(optim->backend);
    gsx_size_t old_rows = 0, new_rows = 0;
    if(optim->param_group_count == 0) return b200_ok();
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    B200_TRY(b200_optim_transition(o, &old_rows, &new_rows, "optimizer param groups must share the same leading extents for resize"));
    if(new_rows != count)
        return gsx_make_error(GSX_ERROR_INVALID_STATE, "optimizer resize expects parameter tensors to already expose the target leading extent");
    return b200_optim_rebuild(o, old_rows, new_rows, NULL);
}

static const gsx_optim_i b200_optim_iface = { b200_optim_destroy,   b200_optim_step_selected, b200_optim_permute,
                                              b200_optim_gather,    b200_optim_resize,        b200_optim_reset_all,
                                              b200_optim_reset_by_index };

static gsx_error b200_create_optim(gsx_backend_t backend, const gsx_optim_desc *desc, gsx_optim_t *out)
{
    b200_backend *be = b200_backend_of(backend);
    b200_optim *o = NULL;
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_optim must be non-null");
    *out = NULL;
    if(desc->algorithm != GSX_OPTIM_ALGORITHM_ADAM) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 implements Adam only");
    o = (b200_optim *)calloc(1, sizeof(*o));
    if(o == NULL) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate the optimizer");
    gsx_error e = gsx_optim_base_init(&o->base, &b200_optim_iface, backend, desc);
    if(!gsx_error_is_success(e)) {
        free(o);
        return e;
    }
    const gsx_index_t ng = o->base.param_group_count;
    o->m1 = (float **)calloc((size_t)ng, sizeof(float *));
    o->m2 = (float **)calloc((size_t)ng, sizeof(float *));
    o->counts = (uint64_t *)calloc((size_t)ng, sizeof(uint64_t));
    o->steps = (uint64_t *)calloc((size_t)ng, sizeof(uint64_t));
    o->rows = (uint64_t *)calloc((size_t)ng, sizeof(uint64_t));
    if(o->m1 == NULL || o->m2 == NULL || o->counts == NULL || o->steps == NULL || o->rows == NULL) {
        b200_optim_free_state(o);
        gsx_optim_base_deinit(&o->base);
        free(o);
        return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate optimizer state records");
    }
    cudaError_t ce = cudaSetDevice(be->ordinal);
    for(gsx_index_t i = 0; i < ng && ce == cudaSuccess; ++i) {
        const gsx_optim_param_group_desc *pg = &o->base.param_groups[i];
        if(pg->parameter->data_type != GSX_DATA_TYPE_F32 || b200_tensor_f32(pg->parameter) == NULL) {
            b200_optim_free_state(o);
            gsx_optim_base_deinit(&o->base);
            free(o);
            return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 Adam requires float32 device parameters");
        }
        o->counts[i] = pg->parameter->size_bytes / sizeof(float);
        o->rows[i] = b200_rows_of(pg->parameter);
        const size_t bytes = (size_t)(o->counts[i] ? o->counts[i] : 1) * sizeof(float);
        ce = cudaMalloc((void **)&o->m1[i], bytes);
        if(ce == cudaSuccess) ce = cudaMalloc((void **)&o->m2[i], bytes);
        if(ce == cudaSuccess) ce = cudaMemsetAsync(o->m1[i], 0, bytes, be->stream);
        if(ce == cudaSuccess) ce = cudaMemsetAsync(o->m2[i], 0, bytes, be->stream);
    }
    if(ce != cudaSuccess) {
        b200_optim_free_state(o);
        gsx_optim_base_deinit(&o->base);
        free(o);
        return b200_cuda_error(ce, "optimizer state allocation failed");
    }
    *out = &o->base;
    return b200_ok();
}

/* ------------------------------------------------------------------------------------------ */
/* backend interface */

static gsx_error b200_backend_free(gsx_backend_t backend)
{
    b200_backend *be = b200_backend_of(backend);
    if(be->base.live_buffer_count > 0 || be->base.live_arena_count > 0)
        return gsx_make_error(GSX_ERROR_INVALID_STATE, "backend has live buffers or arenas");
    if(be->base.live_renderer_count > 0 || be->base.live_loss_count > 0 || be->base.live_optim_count > 0 ||
       be->base.live_adc_count > 0 || be->base.live_async_dl_count > 0)
        return gsx_make_error(GSX_ERROR_INVALID_STATE, "backend has live renderers, losses, optimizers, adcs, or async dataloaders");
    cudaSetDevice(be->ordinal);
    cudaStreamSynchronize(be->stream);
    if(be->finite_word) cudaFree(be->finite_word);
    cudaStreamDestroy(be->stream);
    free(be);
    return b200_ok();
}

static gsx_error b200_backend_get_info(gsx_backend_t backend, gsx_backend_info *out)
{
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_info must be non-null");
    out->backend_type = GSX_BACKEND_TYPE_CUDA;
    out->device = backend->device;
    return b200_ok();
}

static gsx_error b200_backend_get_caps(gsx_backend_t backend, gsx_backend_capabilities *out)
{
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_capabilities must be non-null");
    *out = b200_backend_of(backend)->caps;
    return b200_ok();
}

static gsx_error b200_backend_major_stream(gsx_backend_t backend, void **out)
{
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_stream must be non-null");
    *out = (void *)b200_backend_of(backend)->stream;
    return b200_ok();
}

static gsx_error b200_backend_sync(gsx_backend_t backend)
{
    b200_backend *be = b200_backend_of(backend);
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    return b200_sync(be);
}

static gsx_error b200_backend_count_types(gsx_backend_t backend, gsx_index_t *out)
{
    (void)backend;
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_count must be non-null");
    *out = 2;
    return b200_ok();
}

static gsx_error b200_backend_get_type(gsx_backend_t backend, gsx_index_t index, gsx_backend_buffer_type_t *out)
{
    b200_backend *be = b200_backend_of(backend);
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_buffer_type must be non-null");
    if(index < 0 || index > 1) return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "buffer type index out of range");
    *out = index == 0 ? &be->device_type.base : &be->pinned_type.base;
    return b200_ok();
}

static gsx_error b200_backend_find_type(gsx_backend_t backend, gsx_backend_buffer_type_class cls, gsx_backend_buffer_type_t *out)
{
    b200_backend *be = b200_backend_of(backend);
    if(out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_buffer_type must be non-null");
    if(cls == GSX_BACKEND_BUFFER_TYPE_DEVICE) *out = &be->device_type.base;
    else if(cls == GSX_BACKEND_BUFFER_TYPE_HOST_PINNED) *out = &be->pinned_type.base;
    else return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 backend offers device and pinned-host buffers");
    return b200_ok();
}

static gsx_error b200_backend_unary_ws(gsx_backend_t b, gsx_backend_buffer_type_class c, gsx_data_type d, gsx_index_t xr,
                                       const gsx_index_t *xs, gsx_index_t orr, const gsx_index_t *os, gsx_index_t a,
                                       gsx_impl_unary_reduce_op op, gsx_size_t *sz, gsx_size_t *al)
{
    (void)b, (void)c, (void)d, (void)xr, (void)xs, (void)orr, (void)os, (void)a, (void)op, (void)sz, (void)al;
    return B200_UNSUPPORTED("tensor reductions");
}

static gsx_error b200_backend_binary_ws(gsx_backend_t b, gsx_backend_buffer_type_class c, gsx_data_type d, gsx_index_t lr,
                                        const gsx_index_t *ls, gsx_index_t rr, const gsx_index_t *rs, gsx_index_t orr,
                                        const gsx_index_t *os, gsx_index_t a, gsx_impl_binary_reduce_op op, gsx_size_t *sz,
                                        gsx_size_t *al)
{
    (void)b, (void)c, (void)d, (void)lr, (void)ls, (void)rr, (void)rs, (void)orr, (void)os, (void)a, (void)op, (void)sz, (void)al;
    return B200_UNSUPPORTED("tensor reductions");
}

/* ------------------------------------------------------------------------------------------ */
/* density control: GSX's default ADC (gsx-cuda/adc.cu:948-1040) with the device stages of
 * libgsx_b200 (gsx_b200_adc_*) and GSX's own gsx_gs_gather / gsx_optim_gather for the structural
 * changes, so the Gaussian set, its auxiliary statistics and the optimizer moments move together. */

typedef struct b200_adc {
    struct gsx_adc base;
} b200_adc;

typedef struct b200_adc_fields {
    float *mean3d, *logscale, *opacity, *rotation, *grad_acc, *visible_counter, *max_screen_radius;
} b200_adc_fields;

static gsx_size_t b200_nonneg(gsx_index_t v) { return v <= 0 ? 0 : (gsx_size_t)v; }

/* refine / reset windows of gsx-cuda/adc.cu:78-110 */
static bool b200_adc_refine_window(const gsx_adc_desc *d, gsx_size_t step)
{
    if(d->refine_every == 0 || step % (gsx_size_t)d->refine_every != 0) return false;
    return step >= b200_nonneg(d->start_refine) && step <= b200_nonneg(d->end_refine);
}

static bool b200_adc_reset_window(const gsx_adc_desc *d, gsx_size_t step)
{
    if(d->reset_every == 0 || step % (gsx_size_t)d->reset_every != 0) return false;
    return step >= b200_nonneg(d->start_refine) && step < b200_nonneg(d->end_refine);
}

static bool b200_adc_optim_enabled(const gsx_adc_request *r) { return r->optim != NULL && r->optim->iface != NULL; }

static gsx_error b200_adc_count(gsx_gs_t gs, gsx_size_t *out)
{
    gsx_gs_info info;
    memset(&info, 0, sizeof(info));
    B200_TRY(gsx_gs_get_info(gs, &info));
    *out = info.count;
    return b200_ok();
}

static gsx_error b200_adc_field(gsx_gs_t gs, gsx_gs_field field, gsx_size_t count, gsx_size_t dim1, bool optional,
                                const char *missing, float **out)
{
    gsx_tensor_t t = NULL;
    *out = NULL;
    if(!gsx_error_is_success(gsx_gs_get_field(gs, field, &t)))
        return optional ? b200_ok() : gsx_make_error(GSX_ERROR_NOT_SUPPORTED, missing);
    if(t->data_type != GSX_DATA_TYPE_F32)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 default adc supports only float32 gs fields");
    B200_TRY(gsx_adc_validate_gs_field_shape(t, count, dim1));
    *out = b200_tensor_f32(t);
    if(*out == NULL) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 default adc requires device-backed gs fields");
    return b200_ok();
}

/* the fields the refine pass reads (gsx-cuda/adc.cu:187-277, same requirements and messages) */
static gsx_error b200_adc_load(gsx_gs_t gs, gsx_size_t n, b200_adc_fields *f)
{
    float *unused = NULL;
    memset(f, 0, sizeof(*f));
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_MEAN3D, n, 3, false, "cuda default adc refine requires GSX_GS_FIELD_MEAN3D access", &f->mean3d));
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_GRAD_ACC, n, 1, true, NULL, &f->grad_acc));
    if(f->grad_acc == NULL)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "cuda default adc refine requires GSX_GS_FIELD_GRAD_ACC auxiliary field");
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_VISIBLE_COUNTER, n, 1, true, NULL, &f->visible_counter));
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_LOGSCALE, n, 3, false, "cuda default adc refine requires GSX_GS_FIELD_LOGSCALE access", &f->logscale));
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_OPACITY, n, 1, false, "cuda default adc refine requires GSX_GS_FIELD_OPACITY access", &f->opacity));
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_ROTATION, n, 4, false, "cuda default adc refine requires GSX_GS_FIELD_ROTATION access", &f->rotation));
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_SH0, n, 3, false, "cuda default adc refine requires GSX_GS_FIELD_SH0 access", &unused));
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_SH1, n, 9, true, NULL, &unused));
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_SH2, n, 15, true, NULL, &unused));
    B200_TRY(b200_adc_field(gs, GSX_GS_FIELD_SH3, n, 21, true, NULL, &unused));
    return b200_adc_field(gs, GSX_GS_FIELD_MAX_SCREEN_RADIUS, n, 1, true, NULL, &f->max_screen_radius);
}

/* a rank-1 int32 index tensor over a fresh buffer of the Gaussian set's buffer type */
static gsx_error b200_adc_index_tensor(gsx_gs_t gs, gsx_size_t count, gsx_backend_buffer_t *buf, struct gsx_tensor *t)
{
    gsx_tensor_t mean3d = NULL;
    gsx_backend_buffer_desc bd;
    if(count == 0 || count > (gsx_size_t)INT32_MAX) return gsx_make_error(GSX_ERROR_OUT_OF_RANGE, "index count exceeds supported int32 range");
    B200_TRY(gsx_gs_get_field(gs, GSX_GS_FIELD_MEAN3D, &mean3d));
    memset(&bd, 0, sizeof(bd));
    bd.buffer_type = mean3d->backing_buffer->buffer_type;
    bd.size_bytes = count * sizeof(int32_t);
    bd.alignment_bytes = sizeof(int32_t);
    B200_TRY(gsx_backend_buffer_init(buf, &bd));
    memset(t, 0, sizeof(*t));
    t->arena = mean3d->arena;
    t->backing_buffer = *buf;
    t->size_bytes = bd.size_bytes;
    t->alloc_span_bytes = bd.size_bytes;
    t->requested_alignment_bytes = sizeof(int32_t);
    t->effective_alignment_bytes = sizeof(int32_t);
    t->alloc_end_bytes = bd.size_bytes;
    t->rank = 1;
    t->shape[0] = (gsx_index_t)count;
    t->data_type = GSX_DATA_TYPE_I32;
    t->storage_format = GSX_STORAGE_FORMAT_CHW;
    return b200_ok();
}

/* the Gaussian set and the optimizer state gathered by one index tensor (adc.cu:398-421) */
static gsx_error b200_adc_gather(const gsx_adc_request *r, gsx_tensor_t index)
{
    B200_TRY(gsx_gs_gather(r->gs, index));
    if(b200_adc_optim_enabled(r)) {
        B200_TRY(gsx_optim_rebind_param_groups_from_gs(r->optim, r->gs));
        B200_TRY(gsx_optim_gather(r->optim, index));
    }
    return b200_ok();
}

typedef struct b200_adc_scratch {
    uint8_t *flags;
    int32_t *list;
    uint32_t *words;
    uint32_t *counts;
} b200_adc_scratch;

static void b200_adc_scratch_free(b200_adc_scratch *s)
{
    if(s->flags) cudaFree(s->flags);
    if(s->list) cudaFree(s->list);
    if(s->words) cudaFree(s->words);
    if(s->counts) cudaFree(s->counts);
    memset(s, 0, sizeof(*s));
}

static gsx_error b200_adc_scratch_alloc(b200_adc_scratch *s, gsx_size_t n)
{
    memset(s, 0, sizeof(*s));
    cudaError_t e = cudaMalloc((void **)&s->flags, (size_t)n);
    if(e == cudaSuccess) e = cudaMalloc((void **)&s->list, (size_t)n * sizeof(int32_t));
    if(e == cudaSuccess) e = cudaMalloc((void **)&s->words, (size_t)gsx_b200_adc_scratch_words(n) * sizeof(uint32_t));
    if(e == cudaSuccess) e = cudaMalloc((void **)&s->counts, 2 * sizeof(uint32_t));
    if(e != cudaSuccess) b200_adc_scratch_free(s);
    return b200_cuda_error(e, "adc scratch allocation failed");
}

/* growth (duplicate / split) then prune, gsx-cuda/adc.cu:707-946 */
static gsx_error b200_adc_refine_inner(const gsx_adc_desc *d, b200_backend *be, const gsx_adc_request *r, gsx_adc_result *res,
                                       b200_adc_scratch *sc, gsx_backend_buffer_t *ibuf)
{
    b200_adc_fields f;
    struct gsx_tensor itensor;
    gsx_size_t n0 = 0, n1 = 0, budget = 0, max_cap = b200_nonneg(d->max_num_gaussians);
    uint32_t counts[2] = { 0, 0 };
    B200_TRY(b200_adc_count(r->gs, &n0));
    if(n0 == 0) return b200_ok();
    B200_TRY(b200_adc_load(r->gs, n0, &f));
    budget = max_cap > n0 ? max_cap - n0 : 0;
    if(budget > 0) {
        gsx_size_t grow = 0, split = 0;
        B200_TRY(b200_adc_scratch_alloc(sc, n0));
        B200_TRY(b200_lib_error(gsx_b200_adc_select_growth(n0, f.grad_acc, f.visible_counter, f.logscale, d->duplicate_grad_threshold,
                                                           d->duplicate_scale_threshold, r->scene_scale, budget, sc->flags, sc->list,
                                                           sc->words, sc->counts, be->stream),
                                "gsx_b200_adc_select_growth failed"));
        B200_TRY(b200_cuda_error(cudaMemcpyAsync(counts, sc->counts, sizeof(counts), cudaMemcpyDeviceToHost, be->stream), "D2H failed"));
        B200_TRY(b200_sync(be));
        grow = counts[0] < budget ? counts[0] : budget;
        split = counts[1];
        if(grow > 0) {
            int32_t *ix = NULL;
            B200_TRY(b200_adc_index_tensor(r->gs, n0 + grow, ibuf, &itensor));
            ix = b200_tensor_i32(&itensor);
            if(ix == NULL) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 default adc requires device-backed gs fields");
            B200_TRY(b200_lib_error(gsx_b200_iota_i32(ix, n0, be->stream), "gsx_b200_iota_i32 failed"));
            B200_TRY(b200_cuda_error(cudaMemcpyAsync(ix + n0, sc->list, (size_t)grow * sizeof(int32_t), cudaMemcpyDeviceToDevice, be->stream),
                                     "cudaMemcpyAsync failed"));
            B200_TRY(b200_adc_gather(r, &itensor));
            B200_TRY(gsx_backend_buffer_free(*ibuf));
            *ibuf = NULL;
            B200_TRY(b200_adc_count(r->gs, &n1));
            if(n1 != n0 + grow) return gsx_make_error(GSX_ERROR_INVALID_STATE, "cuda default adc growth produced unexpected gaussian count");
            if(b200_adc_optim_enabled(r)) B200_TRY(gsx_optim_resize(r->optim, n1));
            B200_TRY(b200_adc_load(r->gs, n1, &f));
            B200_TRY(b200_lib_error(gsx_b200_adc_apply_split(grow, sc->list, sc->flags, n0, d->seed, r->global_step, f.mean3d, f.logscale,
                                                             f.opacity, f.rotation, be->stream),
                                    "gsx_b200_adc_apply_split failed"));
            res->duplicated_count += grow - split;
            res->grown_count += split;
            res->mutated = true;
        }
        B200_TRY(b200_sync(be));
        b200_adc_scratch_free(sc);
    }
    B200_TRY(b200_adc_count(r->gs, &n1));
    if(n1 == 0) return b200_ok();
    B200_TRY(b200_adc_load(r->gs, n1, &f));
    B200_TRY(b200_adc_scratch_alloc(sc, n1));
    B200_TRY(b200_lib_error(gsx_b200_adc_select_keep(n1, f.opacity, f.logscale, f.rotation, f.max_screen_radius, n0,
                                                     r->global_step > b200_nonneg(d->reset_every) ? 1 : 0,
                                                     d->pruning_opacity_threshold, d->max_world_scale, d->max_screen_scale,
                                                     r->scene_scale, sc->flags, sc->list, sc->words, sc->counts, be->stream),
                            "gsx_b200_adc_select_keep failed"));
    B200_TRY(b200_cuda_error(cudaMemcpyAsync(counts, sc->counts, sizeof(uint32_t), cudaMemcpyDeviceToHost, be->stream), "D2H failed"));
    B200_TRY(b200_sync(be));
    {
        const gsx_size_t keep = counts[0] == 0 ? 1 : counts[0];
        if(keep < n1) {
            int32_t *ix = NULL;
            B200_TRY(b200_adc_index_tensor(r->gs, keep, ibuf, &itensor));
            ix = b200_tensor_i32(&itensor);
            if(ix == NULL) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 default adc requires device-backed gs fields");
            /* nothing kept: the reference keeps row 0 */
            if(counts[0] == 0) B200_TRY(b200_cuda_error(cudaMemsetAsync(ix, 0, sizeof(int32_t), be->stream), "cudaMemsetAsync failed"));
            else B200_TRY(b200_cuda_error(cudaMemcpyAsync(ix, sc->list, (size_t)keep * sizeof(int32_t), cudaMemcpyDeviceToDevice, be->stream),
                                          "cudaMemcpyAsync failed"));
            B200_TRY(b200_adc_gather(r, &itensor));
            res->pruned_count += n1 - keep;
            res->mutated = true;
        }
    }
    return gsx_gs_zero_aux_tensors(r->gs, GSX_GS_AUX_GRAD_ACC | GSX_GS_AUX_VISIBLE_COUNTER | GSX_GS_AUX_MAX_SCREEN_RADIUS);
}

static gsx_error b200_adc_refine(const gsx_adc_desc *d, b200_backend *be, const gsx_adc_request *r, gsx_adc_result *res)
{
    b200_adc_scratch sc;
    gsx_backend_buffer_t ibuf = NULL;
    gsx_error e;
    memset(&sc, 0, sizeof(sc));
    e = b200_adc_refine_inner(d, be, r, res, &sc, &ibuf);
    if(ibuf != NULL) (void)gsx_backend_buffer_free(ibuf);
    cudaStreamSynchronize(be->stream);
    b200_adc_scratch_free(&sc);
    return e;
}

/* opacity clamp to logit(clamp value) and optimizer reset (gsx-cuda/adc.cu:279-331) */
static gsx_error b200_adc_reset(const gsx_adc_desc *d, const gsx_adc_request *r)
{
    gsx_tensor_t opacity = NULL;
    float lo = -FLT_MAX, hi, p = d->opacity_clamp_value;
    if(!gsx_error_is_success(gsx_gs_get_field(r->gs, GSX_GS_FIELD_OPACITY, &opacity)))
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "cuda default adc reset requires gs opacity access");
    if(opacity->data_type != GSX_DATA_TYPE_F32) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "cuda default adc reset supports only float32 opacity");
    if(p > 1.0f) p = 1.0f;
    if(p < 1e-6f) p = 1e-6f;
    if(p <= 1e-6f) p = 1e-6f;
    if(p >= 1.0f - 1e-6f) p = 1.0f - 1e-6f;
    hi = logf(p / (1.0f - p));
    B200_TRY(gsx_tensor_clamp_inplace(opacity, &lo, &hi));
    if(b200_adc_optim_enabled(r)) B200_TRY(gsx_optim_reset(r->optim));
    return b200_ok();
}

static gsx_error b200_adc_step(gsx_adc_t adc, const gsx_adc_request *request, gsx_adc_result *out)
{
    b200_backend *be = b200_backend_of(adc->backend);
    gsx_size_t before = 0, after = 0;
    if(request == NULL || out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_result must be non-null");
    memset(out, 0, sizeof(*out));
    if(!gsx_error_is_success(b200_adc_count(request->gs, &before)))
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "cuda default adc requires gs info/query support");
    out->gaussians_before = before;
    out->gaussians_after = before;
    B200_TRY(b200_cuda_error(cudaSetDevice(be->ordinal), "cudaSetDevice failed"));
    if(b200_adc_refine_window(&adc->desc, request->global_step)) B200_TRY(b200_adc_refine(&adc->desc, be, request, out));
    if(b200_adc_reset_window(&adc->desc, request->global_step)) {
        B200_TRY(b200_adc_reset(&adc->desc, request));
        out->reset_count = 1;
        out->mutated = true;
    }
    if(!gsx_error_is_success(b200_adc_count(request->gs, &after)))
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "cuda default adc requires gs info/query support");
    out->gaussians_after = after;
    if(after != before) out->mutated = true;
    return b200_ok();
}

static gsx_error b200_adc_destroy(gsx_adc_t adc)
{
    if(adc == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "adc must be non-null");
    gsx_adc_base_deinit(adc);
    free(adc);
    return b200_ok();
}

static const gsx_adc_i b200_adc_iface = { b200_adc_destroy, b200_adc_step };

static gsx_error b200_create_adc(gsx_backend_t backend, const gsx_adc_desc *desc, gsx_adc_t *out)
{
    b200_adc *a = NULL;
    gsx_error e;
    if(out == NULL || desc == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "out_adc and desc must be non-null");
    *out = NULL;
    if(desc->algorithm != GSX_ADC_ALGORITHM_DEFAULT)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "cuda adc currently supports only GSX_ADC_ALGORITHM_DEFAULT");
    a = (b200_adc *)calloc(1, sizeof(*a));
    if(a == NULL) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate the adc");
    e = gsx_adc_base_init(&a->base, &b200_adc_iface, backend, desc);
    if(!gsx_error_is_success(e)) {
        free(a);
        return e;
    }
    *out = &a->base;
    return b200_ok();
}

static gsx_error b200_create_async_dl(gsx_backend_t backend, const gsx_async_dl_desc *desc, gsx_async_dl_t *out)
{
    (void)backend, (void)desc;
    if(out) *out = NULL;
    return B200_UNSUPPORTED("the async dataloader");
}

static const gsx_backend_i b200_backend_iface = {
    b200_backend_free,        b200_backend_get_info, b200_backend_get_caps,   b200_backend_major_stream, b200_backend_sync,
    b200_backend_count_types, b200_backend_get_type, b200_backend_find_type,  b200_backend_unary_ws,     b200_backend_binary_ws,
    b200_create_renderer,     b200_create_loss,      b200_create_optim,       b200_create_adc,           b200_create_async_dl,
};

/* ------------------------------------------------------------------------------------------ */
/* provider */

static gsx_error b200_discover(gsx_backend_provider_t provider, gsx_builtin_registry_state *registry)
{
    int count = 0, k = 0;
    (void)provider;
    cudaError_t e = cudaGetDeviceCount(&count);
    if(e != cudaSuccess || count == 0) return b200_ok();
    for(int ordinal = 0; ordinal < count && k < B200_MAX_DEVICES; ++ordinal) {
        struct cudaDeviceProp prop;
        if(cudaGetDeviceProperties(&prop, ordinal) != cudaSuccess) continue;
        b200_device *d = &b200_devices[k];
        memset(d, 0, sizeof(*d));
        d->base.provider = &b200_provider;
        d->base.info.backend_type = GSX_BACKEND_TYPE_CUDA;
        d->base.info.backend_name = "cuda";
        d->base.info.device_index = k;
        snprintf(d->name, sizeof(d->name), "%s", prop.name);
        d->base.info.name = d->name;
        d->base.info.total_memory_bytes = (gsx_size_t)prop.totalGlobalMem;
        d->ordinal = ordinal;
        B200_TRY(gsx_builtin_registry_append_device(registry, &d->base));
        k += 1;
    }
    return b200_ok();
}

static void b200_init_type(b200_backend *be, b200_buffer_type *t, gsx_backend_buffer_type_class cls, const char *name, gsx_size_t align)
{
    memset(t, 0, sizeof(*t));
    t->base.iface = &b200_type_iface;
    t->base.backend = &be->base;
    t->type_class = cls;
    t->name = name;
    t->alignment = align;
}

static gsx_error b200_create_backend(gsx_backend_device_t device, const gsx_backend_desc *desc, gsx_backend_t *out)
{
    b200_device *d = (b200_device *)device;
    b200_backend *be = NULL;
    if(desc == NULL || out == NULL) return gsx_make_error(GSX_ERROR_INVALID_ARGUMENT, "desc and out_backend must be non-null");
    *out = NULL;
    if(desc->options != NULL || desc->options_size_bytes != 0)
        return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "gsx-b200 backend has no backend-specific options");
    be = (b200_backend *)calloc(1, sizeof(*be));
    if(be == NULL) return gsx_make_error(GSX_ERROR_OUT_OF_MEMORY, "failed to allocate the backend");
    be->base.iface = &b200_backend_iface;
    be->base.provider = &b200_provider;
    be->base.device = device;
    be->ordinal = d->ordinal;
    cudaError_t e = cudaSetDevice(be->ordinal);
    if(e == cudaSuccess) e = cudaStreamCreateWithFlags(&be->stream, cudaStreamNonBlocking);
    if(e == cudaSuccess) e = cudaMalloc((void **)&be->finite_word, sizeof(uint32_t));
    if(e != cudaSuccess) {
        if(be->stream) cudaStreamDestroy(be->stream);
        free(be);
        return b200_cuda_error(e, "backend initialisation failed");
    }
    be->caps.supported_data_types = GSX_DATA_TYPE_FLAG_F32;
    be->caps.supports_async_prefetch = false;
    b200_init_type(be, &be->device_type, GSX_BACKEND_BUFFER_TYPE_DEVICE, "device", 256);
    b200_init_type(be, &be->pinned_type, GSX_BACKEND_BUFFER_TYPE_HOST_PINNED, "host_pinned", 64);
    *out = &be->base;
    return b200_ok();
}

static const gsx_backend_provider_i b200_provider_iface = { b200_discover, b200_create_backend };

gsx_error gsx_cuda_backend_provider_bootstrap(gsx_builtin_registry_state *registry)
{
    int count = 0;
    const cudaError_t e = cudaGetDeviceCount(&count);
    if(e != cudaSuccess || count == 0) return gsx_make_error(GSX_ERROR_NOT_SUPPORTED, "no CUDA devices available");
    b200_provider.iface = &b200_provider_iface;
    b200_provider.backend_type = GSX_BACKEND_TYPE_CUDA;
    b200_provider.backend_name = "cuda";
    B200_TRY(gsx_builtin_registry_append_provider(registry, &b200_provider));
    return b200_provider.iface->discover_devices(&b200_provider, registry);
}
