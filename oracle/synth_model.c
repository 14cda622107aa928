/*
 * Seeded random-init POISDv1 model, written by the test side.
 *
 * TEST INFRASTRUCTURE ONLY.  The bench's reference arm writes its model file
 * with this function so that its process loads nothing of the product
 * (vela_b200/); the product has its own writer (vela_synth_model_write,
 * vela_b200/csrc/synth_model.cpp) for the tests and the bench's own arm.  The
 * two must produce the same bytes for the same seed, which
 * tests/test_synth_model_cpu.py checks on the whole file.
 *
 * Container format (the reference's loader, src/poisd.cpp:17-33): "POISDv1\0",
 * u32 tensor count, then per tensor u16 name length, name bytes, u8 dtype
 * {0 int8, 2 int32, 3 uint8}, u8 rank, u32 dims[rank], little-endian data.
 * Tensor list and shapes: every tensor the reference loader and engine read
 * (src/poisd.cpp:34, src/engine.cu:11-101,389-527) for the SD-2.1 UNet
 * (320/640/1280 channels, 64-dim heads) and the 23-layer 1024-wide text encoder.
 *
 * Values: one splitmix64 stream per tensor group, seeded with the 64-bit FNV-1a
 * hash of the group's name xor the model seed; int8 weights uniform over
 * [-127, 127] (eight bytes per draw, byte value mod 255 minus 127); per output
 * channel m uniform in [16384, 32767], s = 21 + floor(log2(K) / 2) + {0, 1},
 * b uniform in [-50000, 50000]; norms g in 65536 +- 16384, beta in +-8192,
 * eps (the den) 100000; LUTs from their definitions (Q16 logistic and normal
 * CDF on [-16, 16] in steps of 1/64, 2^30 exp(-i/64), Q16 inverse normal CDF of
 * (u + 1/2) / 65536 by bisection).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct { uint64_t state; } sm64_t;

static uint64_t sm64_next(sm64_t* g) {
    uint64_t z = (g->state += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
/* uniform integer in [lo, hi] */
static int64_t sm64_between(sm64_t* g, int64_t lo, int64_t hi) {
    return lo + (int64_t)(sm64_next(g) % (uint64_t)(hi - lo + 1));
}
static sm64_t stream_for(const char* name, uint64_t seed) {
    uint64_t h = 1469598103934665603ull ^ seed;
    for (const unsigned char* c = (const unsigned char*)name; *c; ++c) { h ^= *c; h *= 1099511628211ull; }
    sm64_t g = { h };
    return g;
}

typedef struct { FILE* f; uint32_t count; int failed; uint64_t seed; } out_t;

static void emit(out_t* o, const void* p, size_t n) {
    if (n && fwrite(p, 1, n, o->f) != n) o->failed = 1;
}
static void put_u32(out_t* o, uint32_t v) {
    uint8_t b[4] = { (uint8_t)v, (uint8_t)(v >> 8), (uint8_t)(v >> 16), (uint8_t)(v >> 24) };
    emit(o, b, 4);
}
static void header(out_t* o, const char* name, uint8_t dtype, int rank, const uint32_t* dims) {
    const size_t nl = strlen(name);
    uint8_t b[2] = { (uint8_t)nl, (uint8_t)(nl >> 8) };
    emit(o, b, 2);
    emit(o, name, nl);
    uint8_t t[2] = { dtype, (uint8_t)rank };
    emit(o, t, 2);
    for (int i = 0; i < rank; ++i) put_u32(o, dims[i]);
    o->count++;
}
static void tensor_i32(out_t* o, const char* name, int rank, const uint32_t* dims, const int32_t* v, size_t n) {
    header(o, name, 2, rank, dims);
    for (size_t i = 0; i < n; ++i) put_u32(o, (uint32_t)v[i]);
}
static void vec_i32(out_t* o, const char* name, const int32_t* v, uint32_t n) { tensor_i32(o, name, 1, &n, v, n); }

static char* cat(char* buf, const char* a, const char* b) { snprintf(buf, 256, "%s%s", a, b); return buf; }

/* <base>.w int8 [N, K] and per-column <base>.m / .s / .b, all from the stream of <base> */
static void linear(out_t* o, const char* base, int N, int K) {
    char nm[256];
    sm64_t g = stream_for(base, o->seed);
    const size_t n = (size_t)N * K;
    int8_t* w = (int8_t*)malloc(n ? n : 1);
    for (size_t i = 0; i < n; i += 8) {
        const uint64_t r = sm64_next(&g);
        for (size_t j = 0; j < 8 && i + j < n; ++j) w[i + j] = (int8_t)((int)((r >> (8 * j)) & 255) % 255 - 127);
    }
    const uint32_t dims[2] = { (uint32_t)N, (uint32_t)K };
    header(o, cat(nm, base, ".w"), 0, 2, dims);
    emit(o, w, n);
    free(w);
    const int s0 = 21 + (int)floor(0.5 * log2((double)K));
    int32_t* m = (int32_t*)malloc(sizeof(int32_t) * 3 * (size_t)N);
    int32_t* s = m + N; int32_t* b = s + N;
    for (int c = 0; c < N; ++c) {
        m[c] = (int32_t)sm64_between(&g, 16384, 32767);
        s[c] = (int32_t)(s0 + sm64_between(&g, 0, 1));
        b[c] = (int32_t)sm64_between(&g, -50000, 50000);
    }
    vec_i32(o, cat(nm, base, ".m"), m, (uint32_t)N);
    vec_i32(o, cat(nm, base, ".s"), s, (uint32_t)N);
    vec_i32(o, cat(nm, base, ".b"), b, (uint32_t)N);
    free(m);
}
static void conv3x3(out_t* o, const char* base, int N, int Cin) { linear(o, base, N, 9 * Cin); }
static void norm(out_t* o, const char* base, int C) {
    char nm[256];
    sm64_t g = stream_for(base, o->seed);
    int32_t* gam = (int32_t*)malloc(sizeof(int32_t) * 2 * (size_t)C);
    int32_t* bet = gam + C;
    for (int c = 0; c < C; ++c) {
        gam[c] = (int32_t)sm64_between(&g, 65536 - 16384, 65536 + 16384);
        bet[c] = (int32_t)sm64_between(&g, -8192, 8192);
    }
    vec_i32(o, cat(nm, base, ".g"), gam, (uint32_t)C);
    vec_i32(o, cat(nm, base, ".beta"), bet, (uint32_t)C);
    const int32_t den = 100000;
    vec_i32(o, cat(nm, base, ".eps"), &den, 1);
    free(gam);
}
static void resnet_block(out_t* o, const char* p, int cin, int cout) {
    char nm[256];
    norm(o, cat(nm, p, ".norm1"), cin);
    conv3x3(o, cat(nm, p, ".conv1"), cout, cin);
    norm(o, cat(nm, p, ".norm2"), cout);
    conv3x3(o, cat(nm, p, ".conv2"), cout, cout);
    if (cin != cout) linear(o, cat(nm, p, ".conv_shortcut"), cout, cin);
}
static void transformer_block(out_t* o, const char* p, int C) {
    char nm[256], tb[256];
    norm(o, cat(nm, p, ".norm"), C);
    linear(o, cat(nm, p, ".proj_in"), C, C);
    linear(o, cat(nm, p, ".proj_out"), C, C);
    cat(tb, p, ".transformer_blocks.0");
    static const char* norms[3] = { ".norm1", ".norm2", ".norm3" };
    for (int i = 0; i < 3; ++i) norm(o, cat(nm, tb, norms[i]), C);
    static const char* sq[4] = { ".attn1.to_q", ".attn1.to_k", ".attn1.to_v", ".attn1.to_out.0" };
    for (int i = 0; i < 4; ++i) linear(o, cat(nm, tb, sq[i]), C, C);
    linear(o, cat(nm, tb, ".attn2.to_q"), C, C);
    linear(o, cat(nm, tb, ".attn2.to_k"), C, 1024);
    linear(o, cat(nm, tb, ".attn2.to_v"), C, 1024);
    linear(o, cat(nm, tb, ".attn2.to_out.0"), C, C);
    linear(o, cat(nm, tb, ".ff.net.0.proj.a"), 4 * C, C);
    linear(o, cat(nm, tb, ".ff.net.0.proj.g"), 4 * C, C);
    linear(o, cat(nm, tb, ".ff.net.2"), C, 4 * C);
}

static double phi_cdf(double x) { return 0.5 * erfc(-x / sqrt(2.0)); }
static double phi_inv(double p) {
    double lo = -40.0, hi = 40.0;
    for (int i = 0; i < 200; ++i) {
        const double mid = 0.5 * (lo + hi);
        if (phi_cdf(mid) < p) lo = mid; else hi = mid;
    }
    return 0.5 * (lo + hi);
}

static void unet(out_t* o) {
    char nm[256], blk[128];
    static const int width[4] = { 320, 640, 1280, 1280 };
    int skip[16], nskip = 0;
    conv3x3(o, "unet.conv_in", 320, 4);
    skip[nskip++] = 320;
    int c = 320;
    for (int i = 0; i < 4; ++i) {
        for (int j = 0; j < 2; ++j) {
            snprintf(blk, sizeof blk, "unet.down_blocks.%d.resnets.%d", i, j);
            resnet_block(o, blk, c, width[i]);
            c = width[i];
            if (i < 3) { snprintf(blk, sizeof blk, "unet.down_blocks.%d.attentions.%d", i, j); transformer_block(o, blk, c); }
            skip[nskip++] = c;
        }
        if (i < 3) {
            snprintf(nm, sizeof nm, "unet.down_blocks.%d.downsamplers.0.conv", i);
            conv3x3(o, nm, c, c);
            skip[nskip++] = c;
        }
    }
    resnet_block(o, "unet.mid_block.resnets.0", 1280, 1280);
    transformer_block(o, "unet.mid_block.attentions.0", 1280);
    resnet_block(o, "unet.mid_block.resnets.1", 1280, 1280);
    static const int up_width[4] = { 1280, 1280, 640, 320 };
    for (int i = 0; i < 4; ++i) {
        for (int j = 0; j < 3; ++j) {
            const int s = skip[--nskip];
            snprintf(blk, sizeof blk, "unet.up_blocks.%d.resnets.%d", i, j);
            resnet_block(o, blk, c + s, up_width[i]);
            c = up_width[i];
            if (i > 0) { snprintf(blk, sizeof blk, "unet.up_blocks.%d.attentions.%d", i, j); transformer_block(o, blk, c); }
        }
        if (i < 3) { snprintf(nm, sizeof nm, "unet.up_blocks.%d.upsamplers.0.conv", i); conv3x3(o, nm, c, c); }
    }
    norm(o, "unet.conv_norm_out", 320);
    conv3x3(o, "unet.conv_out", 4, 320);
}

static void text_encoder(out_t* o) {
    char nm[256], lay[64];
    const int vocab = 49408, width = 1024;
    sm64_t g = stream_for("te.tok", o->seed);
    const size_t n = (size_t)vocab * width;
    int8_t* w = (int8_t*)malloc(n);
    for (size_t i = 0; i < n; ++i) w[i] = (int8_t)sm64_between(&g, -127, 127);
    const uint32_t wd[2] = { (uint32_t)vocab, (uint32_t)width };
    header(o, "te.tok.w", 0, 2, wd);
    emit(o, w, n);
    free(w);
    int32_t* tm = (int32_t*)malloc(sizeof(int32_t) * (2 * (size_t)vocab + 77 * (size_t)width));
    int32_t* ts = tm + vocab; int32_t* pos = ts + vocab;
    for (int v = 0; v < vocab; ++v) { tm[v] = (int32_t)sm64_between(&g, 16384, 32767); ts[v] = 22; }
    for (size_t i = 0; i < 77 * (size_t)width; ++i) pos[i] = (int32_t)sm64_between(&g, -16384, 16384);
    vec_i32(o, "te.tok.m", tm, (uint32_t)vocab);
    vec_i32(o, "te.tok.s", ts, (uint32_t)vocab);
    const uint32_t pd[2] = { 77, (uint32_t)width };
    tensor_i32(o, "te.pos", 2, pd, pos, 77 * (size_t)width);
    free(tm);
    for (int l = 0; l < 23; ++l) {
        snprintf(lay, sizeof lay, "te.layers.%d", l);
        norm(o, cat(nm, lay, ".layer_norm1"), width);
        norm(o, cat(nm, lay, ".layer_norm2"), width);
        static const char* proj[4] = { ".self_attn.q_proj", ".self_attn.k_proj", ".self_attn.v_proj", ".self_attn.out_proj" };
        for (int i = 0; i < 4; ++i) linear(o, cat(nm, lay, proj[i]), width, width);
        linear(o, cat(nm, lay, ".mlp.fc1"), 4 * width, width);
        linear(o, cat(nm, lay, ".mlp.fc2"), width, 4 * width);
    }
    norm(o, "te.final_layer_norm", width);
}

static void tables(out_t* o) {
    int32_t* sig = (int32_t*)malloc(sizeof(int32_t) * (2049 * 2 + 1025 + 65536));
    int32_t* phi = sig + 2049; int32_t* ex = phi + 2049; int32_t* gauss = ex + 1025;
    for (int i = 0; i <= 2048; ++i) {
        const double x = (i - 1024) / 64.0;
        sig[i] = (int32_t)lround(65536.0 / (1.0 + exp(-x)));
        phi[i] = (int32_t)lround(65536.0 * phi_cdf(x));
    }
    for (int i = 0; i <= 1024; ++i) ex[i] = (int32_t)lround(1073741824.0 * exp(-i / 64.0));
    for (int u = 0; u < 65536; ++u) gauss[u] = (int32_t)lround(65536.0 * phi_inv((u + 0.5) / 65536.0));
    vec_i32(o, "lut.sigmoid", sig, 2049);
    vec_i32(o, "lut.phi", phi, 2049);
    vec_i32(o, "lut.exp", ex, 1025);
    vec_i32(o, "lut.gauss", gauss, 65536);
    free(sig);
    const int32_t csig = 957800, ccin = 73343000;     /* sigma_max in Q16, 1/sqrt(sigma^2 + 1) in Q30 */
    vec_i32(o, "c.sig", &csig, 1);
    vec_i32(o, "c.cin", &ccin, 1);
    static const char vocab[] = "vela-b200 synthetic vocabulary";
    static const char merges[] = "vela-b200 synthetic merges";
    uint32_t d = (uint32_t)(sizeof vocab - 1);
    header(o, "tok.vocab", 3, 1, &d);
    emit(o, vocab, d);
    d = (uint32_t)(sizeof merges - 1);
    header(o, "tok.merges", 3, 1, &d);
    emit(o, merges, d);
}

/* 0 on success, -1 if the file cannot be created, -2 on a write error */
int or_synth_model_write(const char* path, uint64_t seed) {
    out_t o;
    o.f = fopen(path, "wb");
    if (!o.f) return -1;
    o.count = 0; o.failed = 0; o.seed = seed;
    static const char magic[8] = { 'P', 'O', 'I', 'S', 'D', 'v', '1', 0 };
    emit(&o, magic, 8);
    put_u32(&o, 0);                 /* tensor count, patched below */
    unet(&o);
    text_encoder(&o);
    tables(&o);
    if (fseek(o.f, 8, SEEK_SET) != 0) o.failed = 1;
    put_u32(&o, o.count);
    if (fclose(o.f) != 0) o.failed = 1;
    return o.failed ? -2 : 0;
}
