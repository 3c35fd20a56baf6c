/* generate_moe.c -- greedy generation from a GGUF model file in plain C, on
 * the library's C ABI alone (include/styx_moe.h, styx_attn.h, styx_gguf.h):
 * what crates/model/examples/generate_moe.rs does through MoeModel::load
 * and forward_token (crates/model/src/moe.rs:550-1108, 1780-2140), for a
 * host that is neither Python nor torch.  Token ids in, token ids out.
 *
 *   generate_moe MODEL.gguf N_PREDICT TOK,TOK,... [N_CTX]
 *
 * Build (next to libstyx_moe.so):
 *   cc -O2 -I include styx_b200/host/generate_moe.c -L styx_b200 -lstyx_moe \
 *      -Wl,-rpath,styx_b200 -o generate_moe
 *
 * Per token: the token id and position uploaded (4 bytes each), the
 * embedding row (styx_get_rows), per layer styx_attn_block then
 * styx_moe_block, the output norm, the LM head GEMV and the greedy pick on
 * the device, and the pick downloaded (4 bytes).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "styx_attn.h"
#include "styx_gguf.h"
#include "styx_moe.h"

#define CK(call)                                                                  \
    do {                                                                          \
        int rc_ = (call);                                                         \
        if (rc_) {                                                                \
            fprintf(stderr, "%s failed (%d): %s\n", #call, rc_, styx_last_error()); \
            exit(1);                                                              \
        }                                                                         \
    } while (0)

static styx_ctx *g_ctx;
static styx_gguf *g_file;

/* a tensor of the file uploaded to HBM */
typedef struct {
    void *dev;
    uint32_t type;
    uint64_t bytes;
    uint64_t dims[4];
    uint32_t n_dims;
} tensor;

static int has_tensor(const char *name) { return styx_gguf_find_tensor(g_file, name) >= 0; }

static tensor upload(const char *name) {
    tensor t;
    memset(&t, 0, sizeof(t));
    int64_t i = styx_gguf_find_tensor(g_file, name);
    if (i < 0) {
        fprintf(stderr, "tensor %s missing\n", name);
        exit(1);
    }
    styx_gguf_tensor_info info;
    const void *data = NULL;
    CK(styx_gguf_tensor(g_file, (uint64_t)i, &info));
    CK(styx_gguf_tensor_data(g_file, (uint64_t)i, &data));
    t.type = info.ggml_type;
    t.bytes = info.size_bytes;
    t.n_dims = info.n_dims < 4 ? info.n_dims : 4;
    for (uint32_t d = 0; d < t.n_dims; d++) t.dims[d] = info.dims[d];
    CK(styx_alloc(g_ctx, t.bytes, STYX_MEM_DEVICE, &t.dev));
    CK(styx_upload(g_ctx, t.dev, 0, data, t.bytes, NULL));
    return t;
}

static uint32_t key_u32(const char *arch, const char *key) {
    char k[256];
    uint32_t v = 0;
    snprintf(k, sizeof(k), "%s.%s", arch, key);
    CK(styx_gguf_get_u32(g_file, k, &v));
    return v;
}

static float key_f32(const char *arch, const char *key) {
    char k[256];
    float v = 0.f;
    snprintf(k, sizeof(k), "%s.%s", arch, key);
    CK(styx_gguf_get_f32(g_file, k, &v));
    return v;
}

static void *dev_alloc(uint64_t bytes) {
    void *p = NULL;
    CK(styx_alloc(g_ctx, bytes, STYX_MEM_DEVICE, &p));
    CK(styx_memset(g_ctx, p, 0, bytes, NULL));
    return p;
}

int main(int argc, char **argv) {
    if (argc < 4) {
        fprintf(stderr, "usage: %s MODEL.gguf N_PREDICT TOK,TOK,... [N_CTX]\n", argv[0]);
        return 2;
    }
    const int n_predict = atoi(argv[2]);
    const int n_ctx = argc > 4 ? atoi(argv[4]) : 4096;
    int prompt[4096], n_prompt = 0;
    for (char *s = strtok(argv[3], ","); s && n_prompt < 4096; s = strtok(NULL, ",")) prompt[n_prompt++] = atoi(s);
    if (n_prompt == 0 || n_predict < 1) {
        fprintf(stderr, "empty prompt or nothing to predict\n");
        return 2;
    }

    CK(styx_gguf_open(argv[1], &g_file));
    CK(styx_init(0, &g_ctx));
    const char *arch_s = NULL;
    uint64_t arch_n = 0;
    CK(styx_gguf_get_str(g_file, "general.architecture", &arch_s, &arch_n));
    char arch[64];
    snprintf(arch, sizeof(arch), "%.*s", (int)arch_n, arch_s);

    /* HParams (moe.rs:550-590) */
    const int n_layers = (int)key_u32(arch, "block_count");
    const int H = (int)key_u32(arch, "embedding_length");
    const int n_heads = (int)key_u32(arch, "attention.head_count");
    const int n_kv = (int)key_u32(arch, "attention.head_count_kv");
    char kl[256];
    snprintf(kl, sizeof(kl), "%s.attention.key_length", arch);
    uint32_t hd_u = 0;
    const int hd = styx_gguf_get_u32(g_file, kl, &hd_u) == 0 ? (int)hd_u : H / n_heads;
    const int E = (int)key_u32(arch, "expert_count");
    const int k = (int)key_u32(arch, "expert_used_count");
    /* expert_feed_forward_length, else the width of ffn_gate_exps (olmoe, qwen2moe) */
    char fk[256];
    snprintf(fk, sizeof(fk), "%s.expert_feed_forward_length", arch);
    uint32_t f_u = 0;
    int F = 0;
    if (styx_gguf_get_u32(g_file, fk, &f_u) == 0) {
        F = (int)f_u;
    } else {
        styx_gguf_tensor_info gi;
        const int64_t gidx = styx_gguf_find_tensor(g_file, "blk.0.ffn_gate_exps.weight");
        if (gidx < 0) {
            fprintf(stderr, "no expert_feed_forward_length key and no ffn_gate_exps tensor\n");
            return 1;
        }
        CK(styx_gguf_tensor(g_file, (uint64_t)gidx, &gi));
        F = (int)gi.dims[1];
    }
    /* ArchCfg.norm_topk (moe.rs:324-361) */
    const int norm_topk = strcmp(arch, "qwen3moe") == 0 || strcmp(arch, "qwen3next") == 0;
    const float eps = key_f32(arch, "attention.layer_norm_rms_epsilon");
    const float rope_base = key_f32(arch, "rope.freq_base");
    const int qk_norm = has_tensor("blk.0.attn_q_norm.weight");

    /* weights (moe.rs:996-1108) */
    tensor embd = upload("token_embd.weight"), onorm = upload("output_norm.weight"), head = upload("output.weight");
    const int n_vocab = (int)embd.dims[1];
    styx_attn_layer *al = calloc((size_t)n_layers, sizeof(*al));
    styx_moe_layer *ml = calloc((size_t)n_layers, sizeof(*ml));
    for (int l = 0; l < n_layers; l++) {
        char n[128];
#define T(field) (snprintf(n, sizeof(n), "blk.%d." field ".weight", l), upload(n))
        tensor an = T("attn_norm"), wq = T("attn_q"), wk = T("attn_k"), wv = T("attn_v"), wo = T("attn_output");
        al[l].attn_norm = an.dev;
        al[l].wq = (styx_dense_tensor){wq.dev, (int32_t)wq.type};
        al[l].wk = (styx_dense_tensor){wk.dev, (int32_t)wk.type};
        al[l].wv = (styx_dense_tensor){wv.dev, (int32_t)wv.type};
        al[l].wo = (styx_dense_tensor){wo.dev, (int32_t)wo.type};
        if (qk_norm) {
            tensor qn = T("attn_q_norm"), kn = T("attn_k_norm");
            al[l].q_norm = qn.dev;
            al[l].k_norm = kn.dev;
        }
        tensor fn = T("ffn_norm"), router = T("ffn_gate_inp");
        tensor g = T("ffn_gate_exps"), u = T("ffn_up_exps"), d = T("ffn_down_exps");
#undef T
        ml[l].ffn_norm = fn.dev;
        ml[l].router = router.dev;
        const tensor *ex[3] = {&g, &u, &d};
        styx_expert_tensor *dst[3] = {&ml[l].gate, &ml[l].up, &ml[l].down};
        for (int j = 0; j < 3; j++) {
            memset(dst[j], 0, sizeof(*dst[j]));
            dst[j]->full = ex[j]->dev;
            dst[j]->slab_bytes = ex[j]->bytes / (uint64_t)E;
            dst[j]->qtype = (int32_t)ex[j]->type;
        }
    }
    styx_gguf_close(g_file);

    /* state and workspaces */
    const styx_attn_dims ad = {H, n_heads, n_kv, hd, qk_norm, eps, rope_base};
    const styx_moe_dims md = {H, F, E, k, norm_topk, eps};
    uint64_t aw_bytes = 0, mw_bytes = 0;
    CK(styx_attn_block_workspace_bytes(&ad, &aw_bytes));
    CK(styx_moe_workspace_bytes(&md, &mw_bytes));
    styx_stream st = NULL;
    CK(styx_stream_create(g_ctx, &st));
    void *aws = dev_alloc(aw_bytes), *mws = dev_alloc(mw_bytes);
    CK(styx_attn_block_workspace_init(g_ctx, st, aws, aw_bytes));
    CK(styx_moe_workspace_init(g_ctx, st, mws, mw_bytes));
    const uint64_t kvd = (uint64_t)n_kv * hd;
    float **kc = calloc((size_t)n_layers, sizeof(float *)), **vc = calloc((size_t)n_layers, sizeof(float *));
    for (int l = 0; l < n_layers; l++) {
        kc[l] = dev_alloc((uint64_t)n_ctx * kvd * 4);
        vc[l] = dev_alloc((uint64_t)n_ctx * kvd * 4);
    }
    float *x = dev_alloc((uint64_t)H * 4), *xn = dev_alloc((uint64_t)H * 4), *logits = dev_alloc((uint64_t)n_vocab * 4);
    int32_t *ids = dev_alloc((uint64_t)n_layers * STYX_IDS_PER_LAYER * 4);
    int32_t *tok = dev_alloc(4), *pos_dev = dev_alloc(4), *next = dev_alloc(4);
    CK(styx_stream_sync(g_ctx, NULL));   /* the uploads and clears above, before work on st */

    /* forward_token: returns the greedy pick of the token at position pos */
    int out[4096], n_out = 0, pos = 0, pick = 0;
    for (int step = 0; step < n_prompt + n_predict - 1 && pos < n_ctx; step++, pos++) {
        const int32_t t = step < n_prompt ? prompt[step] : pick;
        const int32_t p = pos;
        CK(styx_upload(g_ctx, tok, 0, &t, 4, st));
        CK(styx_upload(g_ctx, pos_dev, 0, &p, 4, st));
        CK(styx_get_rows(g_ctx, st, (int)embd.type, embd.dev, n_vocab, H, tok, 1, x));
        for (int l = 0; l < n_layers; l++) {
            CK(styx_attn_block(g_ctx, st, &ad, &al[l], x, pos, pos_dev, kc[l], vc[l], n_ctx, aws, aw_bytes));
            CK(styx_moe_block(g_ctx, st, &md, &ml[l], l, x, ids, NULL, mws, mw_bytes));
        }
        CK(styx_rms_norm(g_ctx, st, x, onorm.dev, eps, H, 1, xn));
        CK(styx_mul_mat_vec(g_ctx, st, (int)head.type, head.dev, n_vocab, H, xn, logits));
        CK(styx_argmax_f32(g_ctx, st, logits, n_vocab, next));
        CK(styx_download(g_ctx, &pick, next, 0, 4, st));
        CK(styx_stream_sync(g_ctx, st));
        if (step >= n_prompt - 1 && n_out < 4096) out[n_out++] = pick;
    }
    CK(styx_check_device_error(g_ctx, st));
    for (int i = 0; i < n_out; i++) printf(i ? ",%d" : "%d", out[i]);
    printf("\n");
    styx_destroy(g_ctx);
    return 0;
}
