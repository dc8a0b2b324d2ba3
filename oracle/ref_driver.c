#define _POSIX_C_SOURCE 200809L
/*
 * Thin driver over the UNMODIFIED reference GSX library's public C API (test infrastructure only).
 *
 * Compiled against the reference's public headers and linked against the library that
 * oracle/Makefile.ref builds from the reference sources (CPU: libgsx_ref_cpu.so; CUDA:
 * libgsx_ref_cuda.so).  It exposes a few host-buffer entry points so that tests can compare the
 * oracle with the reference itself, and so that bench.py's reference arm can time the reference
 * CPU backend's training step through the reference's own public API (the calls mirror
 * gsx-runtime.c:1491-1536: render TRAIN, L1 and SSIM forward/backward, render backward, Adam).
 */
#include <gsx/gsx.h>

#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#define REF_CHECK(expr)                                       \
    do {                                                      \
        gsx_error e__ = (expr);                               \
        if(!gsx_error_is_success(e__)) {                      \
            refdrv_last_message = e__.message ? e__.message : #expr; \
            return (int)e__.code ? (int)e__.code : 255;       \
        }                                                     \
    } while(0)

static const char *refdrv_last_message = "";
static gsx_backend_t refdrv_backend = NULL;
static gsx_backend_buffer_type_t refdrv_device_type = NULL;

const char *refdrv_message(void) { return refdrv_last_message; }

/* backend_type: 0 = CPU, 1 = CUDA */
int refdrv_init(int backend_type)
{
    gsx_backend_device_t device = NULL;
    gsx_backend_desc desc;
    if(refdrv_backend != NULL) return 0;
    REF_CHECK(gsx_backend_registry_init());
    REF_CHECK(gsx_get_backend_device_by_type((gsx_backend_type)backend_type, 0, &device));
    memset(&desc, 0, sizeof(desc));
    desc.device = device;
    REF_CHECK(gsx_backend_init(&refdrv_backend, &desc));
    REF_CHECK(gsx_backend_find_buffer_type(refdrv_backend, GSX_BACKEND_BUFFER_TYPE_DEVICE, &refdrv_device_type));
    return 0;
}

static int refdrv_tensor(gsx_arena_t arena, gsx_tensor_t *out, int rank, const int *shape, const float *host)
{
    gsx_tensor_desc d;
    gsx_size_t bytes = sizeof(float);
    memset(&d, 0, sizeof(d));
    d.rank = rank;
    for(int i = 0; i < rank; ++i) {
        d.shape[i] = shape[i];
        bytes *= (gsx_size_t)shape[i];
    }
    d.data_type = GSX_DATA_TYPE_F32;
    d.storage_format = GSX_STORAGE_FORMAT_CHW;
    d.arena = arena;
    REF_CHECK(gsx_tensor_init(out, &d));
    if(host != NULL) {
        REF_CHECK(gsx_tensor_upload(*out, host, bytes));
    } else {
        REF_CHECK(gsx_tensor_set_zero(*out));
    }
    return 0;
}

static int refdrv_arena(gsx_arena_t *arena, gsx_size_t bytes)
{
    gsx_arena_desc ad;
    memset(&ad, 0, sizeof(ad));
    ad.initial_capacity_bytes = bytes;
    REF_CHECK(gsx_arena_init(arena, refdrv_device_type, &ad));
    return 0;
}

/* ---------------------------------------------------------------- a training session */
typedef struct refdrv_session {
    gsx_arena_t arena;
    gsx_renderer_t renderer;
    gsx_render_context_t rctx;
    gsx_loss_t l1, ssim;
    gsx_loss_context_t l1_ctx, ssim_ctx;
    gsx_optim_t optim;
    gsx_tensor_t params[8], grads[8];
    gsx_tensor_t out_rgb, target, loss_map, grad_rgb;
    gsx_tensor_t aux[4]; /* visible_counter, max_screen_radius, grad_acc, absgrad_acc ([N] f32) */
    int aux_on;
    int borrow; /* borrow_train_state of TRAIN requests */
    gsx_camera_intrinsics intr;
    gsx_camera_pose pose;
    float near_plane, far_plane, bg[3];
    int sh_degree, n_fields;
    int64_t n;
    int width, height;
} refdrv_session;

/*
 * fields: mean3d[N,3], rotation[N,4], logscale[N,3], opacity[N], sh0[N,3] (+ sh1/2/3 when sh_degree > 0).
 * lr[8] per role (mean3d, logscale, rotation, opacity, sh0, sh1, sh2, sh3).  target is CHW [3,H,W].
 */
int refdrv_session_create(refdrv_session **out, int64_t n, const float *mean3d, const float *rotation, const float *logscale,
                          const float *opacity, const float *sh0, const float *sh1, const float *sh2, const float *sh3,
                          int sh_degree, int width, int height, float fx, float fy, float cx, float cy, const float q[4],
                          const float t[3], float near_plane, float far_plane, const float bg[3], const float *target,
                          const float lr[8])
{
    refdrv_session *s = (refdrv_session *)calloc(1, sizeof(refdrv_session));
    gsx_size_t per_g = (3 + 4 + 3 + 1 + 3 + 9 + 15 + 21) * 2 * 4 + 4 * 4 + 64;
    gsx_size_t bytes = (gsx_size_t)n * per_g + (gsx_size_t)width * height * 4 * 16 + (1u << 20);
    const float *pv[8] = { mean3d, logscale, rotation, opacity, sh0, sh1, sh2, sh3 };
    const int cols[8] = { 3, 3, 4, 1, 3, 9, 15, 21 };
    gsx_renderer_desc rd;
    gsx_loss_desc ld;
    gsx_optim_param_group_desc groups[8];
    gsx_optim_desc od;
    if(s == NULL) return 1;
    *out = s;
    s->n = n;
    s->width = width;
    s->height = height;
    s->sh_degree = sh_degree;
    s->n_fields = 5 + sh_degree;
    s->near_plane = near_plane;
    s->far_plane = far_plane;
    memcpy(s->bg, bg, sizeof(s->bg));
    if(refdrv_arena(&s->arena, bytes)) return 1;
    for(int f = 0; f < s->n_fields; ++f) {
        int shape[2] = { (int)n, cols[f] };
        if(f == 3) {
            if(refdrv_tensor(s->arena, &s->params[f], 1, shape, pv[f])) return 1;
            if(refdrv_tensor(s->arena, &s->grads[f], 1, shape, NULL)) return 1;
        } else {
            if(f >= 5) shape[1] = cols[f] / 3;
            int shape3[3] = { (int)n, cols[f] / 3, 3 };
            if(f >= 5) {
                if(refdrv_tensor(s->arena, &s->params[f], 3, shape3, pv[f])) return 1;
                if(refdrv_tensor(s->arena, &s->grads[f], 3, shape3, NULL)) return 1;
            } else {
                if(refdrv_tensor(s->arena, &s->params[f], 2, shape, pv[f])) return 1;
                if(refdrv_tensor(s->arena, &s->grads[f], 2, shape, NULL)) return 1;
            }
        }
    }
    {
        int img[3] = { 3, height, width };
        if(refdrv_tensor(s->arena, &s->out_rgb, 3, img, NULL)) return 1;
        if(refdrv_tensor(s->arena, &s->target, 3, img, target)) return 1;
        if(refdrv_tensor(s->arena, &s->loss_map, 3, img, NULL)) return 1;
        if(refdrv_tensor(s->arena, &s->grad_rgb, 3, img, NULL)) return 1;
    }
    for(int k = 0; k < 4; ++k) {
        int shape[1] = { (int)n };
        if(refdrv_tensor(s->arena, &s->aux[k], 1, shape, NULL)) return 1;
        REF_CHECK(gsx_tensor_set_zero(s->aux[k]));
    }
    memset(&rd, 0, sizeof(rd));
    rd.width = width;
    rd.height = height;
    rd.output_data_type = GSX_DATA_TYPE_F32;
    REF_CHECK(gsx_renderer_init(&s->renderer, refdrv_backend, &rd));
    REF_CHECK(gsx_render_context_init(&s->rctx, s->renderer));
    memset(&ld, 0, sizeof(ld));
    ld.algorithm = GSX_LOSS_ALGORITHM_L1;
    ld.grad_normalization = GSX_LOSS_GRAD_NORMALIZATION_TYPE_MEAN;
    REF_CHECK(gsx_loss_init(&s->l1, refdrv_backend, &ld));
    ld.algorithm = GSX_LOSS_ALGORITHM_SSIM;
    REF_CHECK(gsx_loss_init(&s->ssim, refdrv_backend, &ld));
    REF_CHECK(gsx_loss_context_init(&s->l1_ctx, s->l1));
    REF_CHECK(gsx_loss_context_init(&s->ssim_ctx, s->ssim));
    memset(groups, 0, sizeof(groups));
    for(int f = 0; f < s->n_fields; ++f) {
        groups[f].role = (gsx_optim_param_role)f;
        groups[f].parameter = s->params[f];
        groups[f].gradient = s->grads[f];
        groups[f].learning_rate = lr[f];
        groups[f].beta1 = 0.9f;
        groups[f].beta2 = 0.999f;
        groups[f].epsilon = 1e-8f;
    }
    memset(&od, 0, sizeof(od));
    od.algorithm = GSX_OPTIM_ALGORITHM_ADAM;
    od.param_groups = groups;
    od.param_group_count = s->n_fields;
    REF_CHECK(gsx_optim_init(&s->optim, refdrv_backend, &od));
    memset(&s->intr, 0, sizeof(s->intr));
    s->intr.model = (gsx_camera_model)0;
    s->intr.fx = fx;
    s->intr.fy = fy;
    s->intr.cx = cx;
    s->intr.cy = cy;
    s->intr.width = width;
    s->intr.height = height;
    memset(&s->pose, 0, sizeof(s->pose));
    s->pose.rot.x = q[0];
    s->pose.rot.y = q[1];
    s->pose.rot.z = q[2];
    s->pose.rot.w = q[3];
    s->pose.transl.x = t[0];
    s->pose.transl.y = t[1];
    s->pose.transl.z = t[2];
    return 0;
}

static void refdrv_fill_forward(refdrv_session *s, gsx_render_forward_request *rq, gsx_render_forward_type type)
{
    memset(rq, 0, sizeof(*rq));
    rq->intrinsics = &s->intr;
    rq->pose = &s->pose;
    rq->near_plane = s->near_plane;
    rq->far_plane = s->far_plane;
    rq->background_color.x = s->bg[0];
    rq->background_color.y = s->bg[1];
    rq->background_color.z = s->bg[2];
    rq->precision = GSX_RENDER_PRECISION_FLOAT32;
    rq->sh_degree = s->sh_degree;
    rq->forward_type = type;
    rq->borrow_train_state = type == GSX_RENDER_FORWARD_TYPE_TRAIN && s->borrow;
    rq->gs_mean3d = s->params[0];
    rq->gs_logscale = s->params[1];
    rq->gs_rotation = s->params[2];
    rq->gs_opacity = s->params[3];
    rq->gs_sh0 = s->params[4];
    rq->gs_sh1 = s->sh_degree >= 1 ? s->params[5] : NULL;
    rq->gs_sh2 = s->sh_degree >= 2 ? s->params[6] : NULL;
    rq->gs_sh3 = s->sh_degree >= 3 ? s->params[7] : NULL;
    rq->out_rgb = s->out_rgb;
    if(s->aux_on) {
        rq->gs_visible_counter = s->aux[0];
        rq->gs_max_screen_radius = s->aux[1];
    }
}

/* Bind (on != 0) or unbind the four density-control accumulators on later renders and backwards. */
int refdrv_session_enable_aux(refdrv_session *s, int on)
{
    s->aux_on = on;
    return 0;
}

/* TRAIN requests borrow (on != 0) or clone (on == 0, the default) the Gaussian inputs. */
int refdrv_session_set_borrow(refdrv_session *s, int on)
{
    s->borrow = on;
    return 0;
}

/* Forward INFERENCE render into out_rgb (host CHW). */
int refdrv_session_render(refdrv_session *s, float *out_rgb)
{
    gsx_render_forward_request rq;
    refdrv_fill_forward(s, &rq, GSX_RENDER_FORWARD_TYPE_INFERENCE);
    REF_CHECK(gsx_renderer_render(s->renderer, s->rctx, &rq));
    REF_CHECK(gsx_tensor_download(s->out_rgb, out_rgb, (gsx_size_t)3 * s->width * s->height * 4));
    return 0;
}

/* TRAIN forward + backward with a caller-supplied image gradient; downloads the parameter grads
 * in field order (mean3d, logscale, rotation, opacity, sh0[, sh1..]). */
int refdrv_session_render_backward(refdrv_session *s, const float *grad_rgb, float *out_rgb, float **grad_out)
{
    gsx_render_forward_request rq;
    gsx_render_backward_request bq;
    refdrv_fill_forward(s, &rq, GSX_RENDER_FORWARD_TYPE_TRAIN);
    REF_CHECK(gsx_renderer_render(s->renderer, s->rctx, &rq));
    REF_CHECK(gsx_tensor_upload(s->grad_rgb, grad_rgb, (gsx_size_t)3 * s->width * s->height * 4));
    memset(&bq, 0, sizeof(bq));
    bq.grad_rgb = s->grad_rgb;
    bq.grad_gs_mean3d = s->grads[0];
    bq.grad_gs_logscale = s->grads[1];
    bq.grad_gs_rotation = s->grads[2];
    bq.grad_gs_opacity = s->grads[3];
    bq.grad_gs_sh0 = s->grads[4];
    bq.grad_gs_sh1 = s->sh_degree >= 1 ? s->grads[5] : NULL;
    bq.grad_gs_sh2 = s->sh_degree >= 2 ? s->grads[6] : NULL;
    bq.grad_gs_sh3 = s->sh_degree >= 3 ? s->grads[7] : NULL;
    if(s->aux_on) {
        bq.gs_grad_acc = s->aux[2];
        bq.gs_absgrad_acc = s->aux[3];
    }
    REF_CHECK(gsx_renderer_backward(s->renderer, s->rctx, &bq));
    REF_CHECK(gsx_tensor_download(s->out_rgb, out_rgb, (gsx_size_t)3 * s->width * s->height * 4));
    for(int f = 0; f < s->n_fields; ++f) {
        gsx_size_t bytes = 0;
        REF_CHECK(gsx_tensor_get_size_bytes(s->grads[f], &bytes));
        REF_CHECK(gsx_tensor_download(s->grads[f], grad_out[f], bytes));
    }
    return 0;
}

/* TRAIN forward, then the caller's tensors are overwritten with mutated[f] (host, NULL = unchanged),
 * then the backward of grad_rgb: the ordering of the reference tests BackwardUsesRetainedTrainState and
 * BackwardBorrowedTrainStateTracksInputMutations (tests/cuda_render_runtime.cpp:601-689).  Downloads
 * the parameter gradients in field order. */
int refdrv_session_mutate_backward(refdrv_session *s, const float *grad_rgb, const float **mutated, float **grad_out)
{
    gsx_render_forward_request rq;
    gsx_render_backward_request bq;
    refdrv_fill_forward(s, &rq, GSX_RENDER_FORWARD_TYPE_TRAIN);
    REF_CHECK(gsx_renderer_render(s->renderer, s->rctx, &rq));
    for(int f = 0; f < s->n_fields; ++f) {
        if(mutated[f] == NULL) continue;
        gsx_size_t bytes = 0;
        REF_CHECK(gsx_tensor_get_size_bytes(s->params[f], &bytes));
        REF_CHECK(gsx_tensor_upload(s->params[f], mutated[f], bytes));
    }
    REF_CHECK(gsx_tensor_upload(s->grad_rgb, grad_rgb, (gsx_size_t)3 * s->width * s->height * 4));
    memset(&bq, 0, sizeof(bq));
    bq.grad_rgb = s->grad_rgb;
    bq.grad_gs_mean3d = s->grads[0];
    bq.grad_gs_logscale = s->grads[1];
    bq.grad_gs_rotation = s->grads[2];
    bq.grad_gs_opacity = s->grads[3];
    bq.grad_gs_sh0 = s->grads[4];
    bq.grad_gs_sh1 = s->sh_degree >= 1 ? s->grads[5] : NULL;
    bq.grad_gs_sh2 = s->sh_degree >= 2 ? s->grads[6] : NULL;
    bq.grad_gs_sh3 = s->sh_degree >= 3 ? s->grads[7] : NULL;
    REF_CHECK(gsx_renderer_backward(s->renderer, s->rctx, &bq));
    for(int f = 0; f < s->n_fields; ++f) {
        gsx_size_t bytes = 0;
        REF_CHECK(gsx_tensor_get_size_bytes(s->grads[f], &bytes));
        REF_CHECK(gsx_tensor_download(s->grads[f], grad_out[f], bytes));
    }
    return 0;
}

/* One training step exactly as gsx-runtime.c:1413-1536 orders it (without ADC):
 * zero grads, render TRAIN, loss forward L1 (0.8) and SSIM (0.2), loss backward both,
 * render backward, Adam over every group.  Returns 0 and the wall seconds in *seconds. */
int refdrv_session_step(refdrv_session *s, float l1_weight, float ssim_weight, double *seconds)
{
    struct timespec t0, t1;
    gsx_render_forward_request rq;
    gsx_render_backward_request bq;
    gsx_loss_forward_request lf;
    gsx_loss_backward_request lb;
    gsx_optim_step_request oq;
    clock_gettime(CLOCK_MONOTONIC, &t0);
    for(int f = 0; f < s->n_fields; ++f) REF_CHECK(gsx_tensor_set_zero(s->grads[f]));
    REF_CHECK(gsx_tensor_set_zero(s->loss_map));
    REF_CHECK(gsx_tensor_set_zero(s->grad_rgb));
    refdrv_fill_forward(s, &rq, GSX_RENDER_FORWARD_TYPE_TRAIN);
    REF_CHECK(gsx_renderer_render(s->renderer, s->rctx, &rq));
    memset(&lf, 0, sizeof(lf));
    lf.prediction = s->out_rgb;
    lf.target = s->target;
    lf.loss_map_accumulator = s->loss_map;
    lf.train = true;
    lf.scale = l1_weight;
    REF_CHECK(gsx_loss_forward(s->l1, s->l1_ctx, &lf));
    lf.scale = ssim_weight;
    REF_CHECK(gsx_loss_forward(s->ssim, s->ssim_ctx, &lf));
    memset(&lb, 0, sizeof(lb));
    lb.grad_prediction_accumulator = s->grad_rgb;
    lb.scale = l1_weight;
    REF_CHECK(gsx_loss_backward(s->l1, s->l1_ctx, &lb));
    lb.scale = ssim_weight;
    REF_CHECK(gsx_loss_backward(s->ssim, s->ssim_ctx, &lb));
    memset(&bq, 0, sizeof(bq));
    bq.grad_rgb = s->grad_rgb;
    bq.grad_gs_mean3d = s->grads[0];
    bq.grad_gs_logscale = s->grads[1];
    bq.grad_gs_rotation = s->grads[2];
    bq.grad_gs_opacity = s->grads[3];
    bq.grad_gs_sh0 = s->grads[4];
    bq.grad_gs_sh1 = s->sh_degree >= 1 ? s->grads[5] : NULL;
    bq.grad_gs_sh2 = s->sh_degree >= 2 ? s->grads[6] : NULL;
    bq.grad_gs_sh3 = s->sh_degree >= 3 ? s->grads[7] : NULL;
    REF_CHECK(gsx_renderer_backward(s->renderer, s->rctx, &bq));
    memset(&oq, 0, sizeof(oq));
    oq.force_all = true;
    REF_CHECK(gsx_optim_step(s->optim, &oq));
    REF_CHECK(gsx_backend_major_stream_sync(refdrv_backend));
    clock_gettime(CLOCK_MONOTONIC, &t1);
    if(seconds) *seconds = (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
    return 0;
}

/* Download the current parameter, loss map or rendered image. which: 0..7 params, 8 out_rgb, 9 loss_map, 10 grad_rgb,
 * 11..14 visible_counter, max_screen_radius, grad_acc, absgrad_acc */
int refdrv_session_download(refdrv_session *s, int which, float *dst)
{
    gsx_tensor_t t = which >= 11 ? s->aux[which - 11]
                                 : which < 8 ? s->params[which] : (which == 8 ? s->out_rgb : (which == 9 ? s->loss_map : s->grad_rgb));
    gsx_size_t bytes = 0;
    REF_CHECK(gsx_tensor_get_size_bytes(t, &bytes));
    REF_CHECK(gsx_tensor_download(t, dst, bytes));
    return 0;
}

/* ---------------------------------------------------------------- standalone loss and Adam */
/* algorithm: 0 L1, 1 MSE, 2 SSIM; normalization 0 MEAN, 1 SUM; shape [outer, C, H, W] CHW.
 * loss_map and grad are read, accumulated into by the reference, and written back. */
int refdrv_loss(int algorithm, int normalization, int outer, int channels, int height, int width, const float *pred,
                const float *target, float scale, float *loss_map, float *grad)
{
    gsx_arena_t arena = NULL;
    gsx_loss_t loss = NULL;
    gsx_loss_context_t ctx = NULL;
    gsx_tensor_t tp = NULL, tt = NULL, tl = NULL, tg = NULL;
    gsx_loss_desc ld;
    gsx_loss_forward_request lf;
    gsx_loss_backward_request lb;
    const gsx_size_t n = (gsx_size_t)outer * channels * height * width;
    int shape[4] = { outer, channels, height, width };
    int rc = 0;
    if(refdrv_arena(&arena, n * 4 * 4 + 4096)) return 1;
    if((rc = refdrv_tensor(arena, &tp, 4, shape, pred)) != 0) return rc;
    if((rc = refdrv_tensor(arena, &tt, 4, shape, target)) != 0) return rc;
    if((rc = refdrv_tensor(arena, &tl, 4, shape, loss_map)) != 0) return rc;
    if((rc = refdrv_tensor(arena, &tg, 4, shape, grad)) != 0) return rc;
    memset(&ld, 0, sizeof(ld));
    ld.algorithm = (gsx_loss_algorithm)algorithm;
    ld.grad_normalization = (gsx_loss_grad_normalization_type)normalization;
    REF_CHECK(gsx_loss_init(&loss, refdrv_backend, &ld));
    REF_CHECK(gsx_loss_context_init(&ctx, loss));
    memset(&lf, 0, sizeof(lf));
    lf.prediction = tp;
    lf.target = tt;
    lf.loss_map_accumulator = tl;
    lf.train = true;
    lf.scale = scale;
    REF_CHECK(gsx_loss_forward(loss, ctx, &lf));
    memset(&lb, 0, sizeof(lb));
    lb.grad_prediction_accumulator = tg;
    lb.scale = scale;
    REF_CHECK(gsx_loss_backward(loss, ctx, &lb));
    REF_CHECK(gsx_tensor_download(tl, loss_map, n * 4));
    REF_CHECK(gsx_tensor_download(tg, grad, n * 4));
    gsx_tensor_free(tg);
    gsx_tensor_free(tl);
    gsx_tensor_free(tt);
    gsx_tensor_free(tp);
    gsx_loss_context_free(ctx);
    gsx_loss_free(loss);
    gsx_arena_free(arena);
    return 0;
}

/* `steps` Adam steps on one [n] group with a fixed gradient; param/m state returned in place. */
int refdrv_adam(int64_t n, float *param, const float *grad, int steps, float lr, float beta1, float beta2, float eps,
                float weight_decay, float max_grad)
{
    gsx_arena_t arena = NULL;
    gsx_tensor_t tp = NULL, tg = NULL;
    gsx_optim_t optim = NULL;
    gsx_optim_param_group_desc g;
    gsx_optim_desc od;
    gsx_optim_step_request oq;
    int shape[1] = { (int)n };
    int rc = 0;
    if(refdrv_arena(&arena, (gsx_size_t)n * 8 + 4096)) return 1;
    if((rc = refdrv_tensor(arena, &tp, 1, shape, param)) != 0) return rc;
    if((rc = refdrv_tensor(arena, &tg, 1, shape, grad)) != 0) return rc;
    memset(&g, 0, sizeof(g));
    g.role = GSX_OPTIM_PARAM_ROLE_MEAN3D;
    g.parameter = tp;
    g.gradient = tg;
    g.learning_rate = lr;
    g.beta1 = beta1;
    g.beta2 = beta2;
    g.epsilon = eps;
    g.weight_decay = weight_decay;
    g.max_grad = max_grad;
    memset(&od, 0, sizeof(od));
    od.algorithm = GSX_OPTIM_ALGORITHM_ADAM;
    od.param_groups = &g;
    od.param_group_count = 1;
    REF_CHECK(gsx_optim_init(&optim, refdrv_backend, &od));
    memset(&oq, 0, sizeof(oq));
    oq.force_all = true;
    for(int s = 0; s < steps; ++s) REF_CHECK(gsx_optim_step(optim, &oq));
    REF_CHECK(gsx_tensor_download(tp, param, (gsx_size_t)n * 4));
    gsx_optim_free(optim);
    gsx_tensor_free(tg);
    gsx_tensor_free(tp);
    gsx_arena_free(arena);
    return 0;
}

/* a one-sample 4x4 u8 dataset: the ADC request needs a dataloader and a renderer handle */
static const uint8_t refdrv_tiny_rgb[4 * 4 * 3] = { 0 };
static gsx_error refdrv_ok(void)
{
    gsx_error e;
    e.code = GSX_ERROR_SUCCESS;
    e.message = NULL;
    return e;
}
static gsx_error refdrv_tiny_length(void *o, gsx_size_t *n)
{
    (void)o;
    *n = 1;
    return refdrv_ok();
}
static gsx_error refdrv_tiny_sample(void *o, gsx_size_t i, gsx_dataset_cpu_sample *s)
{
    (void)o, (void)i;
    memset(s, 0, sizeof(*s));
    s->intrinsics.fx = s->intrinsics.fy = 4.0f;
    s->intrinsics.cx = s->intrinsics.cy = 2.0f;
    s->intrinsics.width = s->intrinsics.height = 4;
    s->pose.rot.w = 1.0f;
    s->rgb_data = refdrv_tiny_rgb;
    return refdrv_ok();
}
static void refdrv_tiny_release(void *o, gsx_dataset_cpu_sample *s) { (void)o, (void)s; }

/* ---------------------------------------------------------------- density control
 * One GSX density-control step through the public API, as the runtime drives it
 * (gsx-runtime.c ADC stage): a gsx_gs holding `n` Gaussians (mean3d, logscale, rotation, opacity,
 * sh0 and the grad_acc / visible_counter / max_screen_radius statistics), an Adam optimizer bound to
 * its fields and stepped once with the given gradients (so the moments are non-trivial), then
 * gsx_adc_step with the default algorithm, then one more Adam step with every gradient = 1 (so the
 * gathered moments show in the parameters).
 *   fparams: pruning_opacity_threshold, opacity_clamp_value, max_world_scale, max_screen_scale,
 *            duplicate_grad_threshold, duplicate_scale_threshold, scene_scale
 *   iparams: refine_every, start_refine, end_refine, max_num_gaussians, reset_every, seed, global_step
 *   grads:   gradients of mean3d, logscale, rotation, opacity, sh0 for the first Adam step
 *   result:  gaussians_before, gaussians_after, pruned, duplicated, grown, reset_count, mutated
 *   out_after_adc / out_final: the five fields (same layout as the inputs, `cap` Gaussians of room),
 *   after the ADC step and after the final Adam step; out_aux: the three statistics after ADC. */
int refdrv_adc_run(int64_t n, const float *mean3d, const float *logscale, const float *rotation, const float *opacity,
                   const float *sh0, const float *grad_acc, const float *visible_counter, const float *max_screen_radius,
                   const float *const *grads, const float *fparams, const int64_t *iparams, int64_t *result, int64_t cap,
                   float *const *out_after_adc, float *const *out_final, float *const *out_aux)
{
    static const int cols[5] = { 3, 3, 4, 1, 3 };
    const float *in[5] = { mean3d, logscale, rotation, opacity, sh0 };
    const float *aux_in[3] = { grad_acc, visible_counter, max_screen_radius };
    const gsx_gs_field aux_field[3] = { GSX_GS_FIELD_GRAD_ACC, GSX_GS_FIELD_VISIBLE_COUNTER, GSX_GS_FIELD_MAX_SCREEN_RADIUS };
    gsx_gs_t gs = NULL;
    gsx_gs_desc gd;
    gsx_optim_t optim = NULL;
    gsx_optim_param_group_desc groups[5];
    gsx_optim_desc od;
    gsx_optim_step_request oq;
    gsx_adc_t adc = NULL;
    gsx_adc_desc ad;
    gsx_adc_request rq;
    gsx_adc_result res;
    gsx_gs_info info;
    float *ones = NULL;
    gsx_dataset_t ds = NULL;
    gsx_dataset_desc dsd;
    gsx_dataloader_t dl = NULL;
    gsx_dataloader_desc dld;
    gsx_renderer_t ren = NULL;
    gsx_renderer_desc rd;
    memset(&dsd, 0, sizeof(dsd));
    dsd.image_data_type = GSX_DATA_TYPE_U8;
    dsd.width = dsd.height = 4;
    dsd.has_rgb = true;
    dsd.get_length = refdrv_tiny_length;
    dsd.get_sample = refdrv_tiny_sample;
    dsd.release_sample = refdrv_tiny_release;
    REF_CHECK(gsx_dataset_init(&ds, &dsd));
    memset(&dld, 0, sizeof(dld));
    dld.image_data_type = GSX_DATA_TYPE_F32;
    REF_CHECK(gsx_dataloader_init(&dl, refdrv_backend, ds, &dld));
    memset(&rd, 0, sizeof(rd));
    rd.width = rd.height = 4;
    rd.output_data_type = GSX_DATA_TYPE_F32;
    REF_CHECK(gsx_renderer_init(&ren, refdrv_backend, &rd));
    memset(&gd, 0, sizeof(gd));
    gd.buffer_type = refdrv_device_type;
    gd.count = (gsx_size_t)n;
    gd.aux_flags = GSX_GS_AUX_GRAD_ACC | GSX_GS_AUX_VISIBLE_COUNTER | GSX_GS_AUX_MAX_SCREEN_RADIUS;
    REF_CHECK(gsx_gs_init(&gs, &gd));
    for(int f = 0; f < 5; ++f) {
        gsx_tensor_t t = NULL;
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)f, &t));
        REF_CHECK(gsx_tensor_upload(t, in[f], (gsx_size_t)n * cols[f] * sizeof(float)));
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)(GSX_GS_FIELD_GRAD_MEAN3D + f), &t));
        REF_CHECK(gsx_tensor_upload(t, grads[f], (gsx_size_t)n * cols[f] * sizeof(float)));
    }
    for(int k = 0; k < 3; ++k) {
        gsx_tensor_t t = NULL;
        REF_CHECK(gsx_gs_get_field(gs, aux_field[k], &t));
        REF_CHECK(gsx_tensor_upload(t, aux_in[k], (gsx_size_t)n * sizeof(float)));
    }
    memset(groups, 0, sizeof(groups));
    for(int f = 0; f < 5; ++f) {
        groups[f].role = (gsx_optim_param_role)f;
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)f, &groups[f].parameter));
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)(GSX_GS_FIELD_GRAD_MEAN3D + f), &groups[f].gradient));
        groups[f].learning_rate = f == 0 ? 1e-3f : 1e-2f;
        groups[f].beta1 = 0.9f;
        groups[f].beta2 = 0.999f;
        groups[f].epsilon = 1e-8f;
    }
    memset(&od, 0, sizeof(od));
    od.algorithm = GSX_OPTIM_ALGORITHM_ADAM;
    od.param_groups = groups;
    od.param_group_count = 5;
    REF_CHECK(gsx_optim_init(&optim, refdrv_backend, &od));
    memset(&oq, 0, sizeof(oq));
    oq.force_all = true;
    REF_CHECK(gsx_optim_step(optim, &oq));

    memset(&ad, 0, sizeof(ad));
    ad.algorithm = GSX_ADC_ALGORITHM_DEFAULT;
    ad.pruning_opacity_threshold = fparams[0];
    ad.opacity_clamp_value = fparams[1];
    ad.max_world_scale = fparams[2];
    ad.max_screen_scale = fparams[3];
    ad.duplicate_grad_threshold = fparams[4];
    ad.duplicate_scale_threshold = fparams[5];
    ad.refine_every = (gsx_index_t)iparams[0];
    ad.start_refine = (gsx_index_t)iparams[1];
    ad.end_refine = (gsx_index_t)iparams[2];
    ad.max_num_gaussians = (gsx_index_t)iparams[3];
    ad.reset_every = (gsx_index_t)iparams[4];
    ad.seed = (gsx_size_t)iparams[5];
    REF_CHECK(gsx_adc_init(&adc, refdrv_backend, &ad));
    memset(&rq, 0, sizeof(rq));
    rq.gs = gs;
    rq.optim = optim;
    rq.dataloader = dl;
    rq.renderer = ren;
    rq.global_step = (gsx_size_t)iparams[6];
    rq.scene_scale = fparams[6];
    memset(&res, 0, sizeof(res));
    REF_CHECK(gsx_adc_step(adc, &rq, &res));
    result[0] = (int64_t)res.gaussians_before;
    result[1] = (int64_t)res.gaussians_after;
    result[2] = (int64_t)res.pruned_count;
    result[3] = (int64_t)res.duplicated_count;
    result[4] = (int64_t)res.grown_count;
    result[5] = (int64_t)res.reset_count;
    result[6] = res.mutated ? 1 : 0;
    memset(&info, 0, sizeof(info));
    REF_CHECK(gsx_gs_get_info(gs, &info));
    if((int64_t)info.count > cap) return 254;
    for(int f = 0; f < 5; ++f) {
        gsx_tensor_t t = NULL;
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)f, &t));
        REF_CHECK(gsx_tensor_download(t, out_after_adc[f], (gsx_size_t)info.count * cols[f] * sizeof(float)));
    }
    for(int k = 0; k < 3; ++k) {
        gsx_tensor_t t = NULL;
        REF_CHECK(gsx_gs_get_field(gs, aux_field[k], &t));
        REF_CHECK(gsx_tensor_download(t, out_aux[k], (gsx_size_t)info.count * sizeof(float)));
    }
    /* one more Adam step with unit gradients: the moments the ADC step carried show in the parameters */
    ones = (float *)malloc((size_t)(info.count ? info.count : 1) * 4 * sizeof(float));
    if(ones == NULL) return 253;
    for(gsx_size_t i = 0; i < info.count * 4; ++i) ones[i] = 1.0f;
    for(int f = 0; f < 5; ++f) {
        gsx_tensor_t t = NULL;
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)(GSX_GS_FIELD_GRAD_MEAN3D + f), &t));
        REF_CHECK(gsx_tensor_upload(t, ones, (gsx_size_t)info.count * cols[f] * sizeof(float)));
    }
    free(ones);
    REF_CHECK(gsx_optim_rebind_param_groups_from_gs(optim, gs));
    REF_CHECK(gsx_optim_step(optim, &oq));
    for(int f = 0; f < 5; ++f) {
        gsx_tensor_t t = NULL;
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)f, &t));
        REF_CHECK(gsx_tensor_download(t, out_final[f], (gsx_size_t)info.count * cols[f] * sizeof(float)));
    }
    REF_CHECK(gsx_backend_major_stream_sync(refdrv_backend));
    REF_CHECK(gsx_adc_free(adc));
    REF_CHECK(gsx_optim_free(optim));
    REF_CHECK(gsx_gs_free(gs));
    REF_CHECK(gsx_renderer_free(ren));
    REF_CHECK(gsx_dataloader_free(dl));
    REF_CHECK(gsx_dataset_free(ds));
    return 0;
}

/* ---------------------------------------------------------------- runtime session
 * GSX's own training loop (gsx_session_step: dataloader -> render TRAIN -> L1 + SSIM -> backward ->
 * Adam -> ADC) over a one-image dataset, `steps` steps.  Inputs as refdrv_adc_run plus the target
 * image (f32 HWC [H,W,3]) and its camera.  Per step: the summed loss map and the Gaussian count;
 * at the end the five fields (`cap` Gaussians of room). */
typedef struct refdrv_fit_data {
    const float *rgb;
    int width, height;
    float fx, fy, cx, cy, q[4], t[3];
} refdrv_fit_data;

static gsx_error refdrv_fit_sample(void *o, gsx_size_t i, gsx_dataset_cpu_sample *s)
{
    const refdrv_fit_data *d = (const refdrv_fit_data *)o;
    (void)i;
    memset(s, 0, sizeof(*s));
    s->intrinsics.fx = d->fx;
    s->intrinsics.fy = d->fy;
    s->intrinsics.cx = d->cx;
    s->intrinsics.cy = d->cy;
    s->intrinsics.width = d->width;
    s->intrinsics.height = d->height;
    s->pose.rot.x = d->q[0];
    s->pose.rot.y = d->q[1];
    s->pose.rot.z = d->q[2];
    s->pose.rot.w = d->q[3];
    s->pose.transl.x = d->t[0];
    s->pose.transl.y = d->t[1];
    s->pose.transl.z = d->t[2];
    s->rgb_data = d->rgb;
    return refdrv_ok();
}

int refdrv_session_fit(int64_t n, const float *mean3d, const float *logscale, const float *rotation, const float *opacity,
                       const float *sh0, const float *target_hwc, int width, int height, const float *cam /* fx fy cx cy q4 t3 */,
                       const float *fparams, const int64_t *iparams, int64_t steps, float *loss_out, int64_t *count_out,
                       int64_t cap, float *const *out_fields)
{
    static const int cols[5] = { 3, 3, 4, 1, 3 };
    const float *in[5] = { mean3d, logscale, rotation, opacity, sh0 };
    refdrv_fit_data data;
    gsx_dataset_t ds = NULL;
    gsx_dataset_desc dsd;
    gsx_dataloader_t dl = NULL;
    gsx_dataloader_desc dld;
    gsx_renderer_t ren = NULL;
    gsx_renderer_desc rd;
    gsx_gs_t gs = NULL;
    gsx_gs_desc gd;
    gsx_optim_t optim = NULL;
    gsx_optim_param_group_desc groups[5];
    gsx_optim_desc od;
    gsx_adc_t adc = NULL;
    gsx_adc_desc ad;
    gsx_gs_aux_flags aux_flags = 0;
    gsx_loss_t l1 = NULL, ssim = NULL;
    gsx_loss_context_t l1c = NULL, ssimc = NULL;
    gsx_loss_desc ld;
    gsx_loss_item items[2];
    gsx_session_t session = NULL;
    gsx_session_desc sd;
    float *host = (float *)malloc((size_t)width * height * 3 * sizeof(float));
    if(host == NULL) return 253;
    data.rgb = target_hwc;
    data.width = width;
    data.height = height;
    data.fx = cam[0];
    data.fy = cam[1];
    data.cx = cam[2];
    data.cy = cam[3];
    memcpy(data.q, cam + 4, sizeof(data.q));
    memcpy(data.t, cam + 8, sizeof(data.t));
    memset(&dsd, 0, sizeof(dsd));
    dsd.object = &data;
    dsd.image_data_type = GSX_DATA_TYPE_F32;
    dsd.width = width;
    dsd.height = height;
    dsd.has_rgb = true;
    dsd.get_length = refdrv_tiny_length;
    dsd.get_sample = refdrv_fit_sample;
    dsd.release_sample = refdrv_tiny_release;
    REF_CHECK(gsx_dataset_init(&ds, &dsd));
    memset(&dld, 0, sizeof(dld));
    dld.image_data_type = GSX_DATA_TYPE_F32;
    REF_CHECK(gsx_dataloader_init(&dl, refdrv_backend, ds, &dld));
    memset(&rd, 0, sizeof(rd));
    rd.width = width;
    rd.height = height;
    rd.output_data_type = GSX_DATA_TYPE_F32;
    REF_CHECK(gsx_renderer_init(&ren, refdrv_backend, &rd));

    memset(&ad, 0, sizeof(ad));
    ad.algorithm = GSX_ADC_ALGORITHM_DEFAULT;
    ad.pruning_opacity_threshold = fparams[0];
    ad.opacity_clamp_value = fparams[1];
    ad.max_world_scale = fparams[2];
    ad.max_screen_scale = fparams[3];
    ad.duplicate_grad_threshold = fparams[4];
    ad.duplicate_scale_threshold = fparams[5];
    ad.refine_every = (gsx_index_t)iparams[0];
    ad.start_refine = (gsx_index_t)iparams[1];
    ad.end_refine = (gsx_index_t)iparams[2];
    ad.max_num_gaussians = (gsx_index_t)iparams[3];
    ad.reset_every = (gsx_index_t)iparams[4];
    ad.seed = (gsx_size_t)iparams[5];
    REF_CHECK(gsx_adc_init(&adc, refdrv_backend, &ad));
    REF_CHECK(gsx_adc_get_gs_aux_fields(adc, &aux_flags));

    memset(&gd, 0, sizeof(gd));
    gd.buffer_type = refdrv_device_type;
    gd.count = (gsx_size_t)n;
    gd.aux_flags = aux_flags;
    REF_CHECK(gsx_gs_init(&gs, &gd));
    for(int f = 0; f < 5; ++f) {
        gsx_tensor_t t = NULL;
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)f, &t));
        REF_CHECK(gsx_tensor_upload(t, in[f], (gsx_size_t)n * cols[f] * sizeof(float)));
    }
    REF_CHECK(gsx_gs_zero_aux_tensors(gs, aux_flags));
    memset(groups, 0, sizeof(groups));
    for(int f = 0; f < 5; ++f) {
        groups[f].role = (gsx_optim_param_role)f;
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)f, &groups[f].parameter));
        REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)(GSX_GS_FIELD_GRAD_MEAN3D + f), &groups[f].gradient));
        groups[f].learning_rate = f == 0 ? 1.6e-4f : (f == 3 ? 5e-2f : (f == 4 ? 2.5e-3f : (f == 1 ? 5e-3f : 1e-3f)));
        groups[f].beta1 = 0.9f;
        groups[f].beta2 = 0.999f;
        groups[f].epsilon = 1e-15f;
    }
    memset(&od, 0, sizeof(od));
    od.algorithm = GSX_OPTIM_ALGORITHM_ADAM;
    od.param_groups = groups;
    od.param_group_count = 5;
    REF_CHECK(gsx_optim_init(&optim, refdrv_backend, &od));

    memset(&ld, 0, sizeof(ld));
    ld.algorithm = GSX_LOSS_ALGORITHM_L1;
    ld.grad_normalization = GSX_LOSS_GRAD_NORMALIZATION_TYPE_MEAN;
    REF_CHECK(gsx_loss_init(&l1, refdrv_backend, &ld));
    ld.algorithm = GSX_LOSS_ALGORITHM_SSIM;
    REF_CHECK(gsx_loss_init(&ssim, refdrv_backend, &ld));
    REF_CHECK(gsx_loss_context_init(&l1c, l1));
    REF_CHECK(gsx_loss_context_init(&ssimc, ssim));
    items[0].loss = l1;
    items[0].context = l1c;
    items[0].scale = 0.8f;
    items[1].loss = ssim;
    items[1].context = ssimc;
    items[1].scale = 0.2f;

    memset(&sd, 0, sizeof(sd));
    sd.backend = refdrv_backend;
    sd.gs = gs;
    sd.optim = optim;
    sd.renderer = ren;
    sd.train_dataloader = dl;
    sd.adc = adc;
    sd.loss_count = 2;
    sd.loss_items = items;
    sd.render.near_plane = 0.01f;
    sd.render.far_plane = 100.0f;
    sd.render.precision = GSX_RENDER_PRECISION_FLOAT32;
    sd.render.sh_degree_mode = GSX_SESSION_SH_DEGREE_MODE_EXPLICIT;
    sd.render.sh_degree = 0;
    sd.optim_step.force_all = true;
    sd.adc_step.enabled = true;
    sd.adc_step.scene_scale = fparams[6];
    sd.workspace.buffer_type_class = GSX_BACKEND_BUFFER_TYPE_DEVICE;
    sd.workspace.auto_plan = true;
    sd.reporting.retain_loss_map = true;
    REF_CHECK(gsx_session_init(&session, &sd));
    for(int64_t k = 0; k < steps; ++k) {
        gsx_session_outputs outs;
        gsx_gs_info info;
        double sum = 0.0;
        REF_CHECK(gsx_session_step(session));
        memset(&outs, 0, sizeof(outs));
        REF_CHECK(gsx_session_get_last_outputs(session, &outs));
        if(outs.loss_map == NULL) return 252;
        REF_CHECK(gsx_tensor_download(outs.loss_map, host, (gsx_size_t)width * height * 3 * sizeof(float)));
        for(int64_t i = 0; i < (int64_t)width * height * 3; ++i) sum += host[i];
        loss_out[k] = (float)(sum / ((double)width * height * 3));
        memset(&info, 0, sizeof(info));
        REF_CHECK(gsx_gs_get_info(gs, &info));
        count_out[k] = (int64_t)info.count;
    }
    {
        gsx_gs_info info;
        memset(&info, 0, sizeof(info));
        REF_CHECK(gsx_gs_get_info(gs, &info));
        if((int64_t)info.count > cap) return 254;
        for(int f = 0; f < 5; ++f) {
            gsx_tensor_t t = NULL;
            REF_CHECK(gsx_gs_get_field(gs, (gsx_gs_field)f, &t));
            REF_CHECK(gsx_tensor_download(t, out_fields[f], (gsx_size_t)info.count * cols[f] * sizeof(float)));
        }
    }
    free(host);
    REF_CHECK(gsx_backend_major_stream_sync(refdrv_backend));
    REF_CHECK(gsx_session_free(session));
    REF_CHECK(gsx_loss_context_free(l1c));
    REF_CHECK(gsx_loss_context_free(ssimc));
    REF_CHECK(gsx_loss_free(l1));
    REF_CHECK(gsx_loss_free(ssim));
    REF_CHECK(gsx_optim_free(optim));
    REF_CHECK(gsx_adc_free(adc));
    REF_CHECK(gsx_gs_free(gs));
    REF_CHECK(gsx_renderer_free(ren));
    REF_CHECK(gsx_dataloader_free(dl));
    REF_CHECK(gsx_dataset_free(ds));
    return 0;
}
