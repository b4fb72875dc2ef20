// sml-gpu-fwd: the reference's GPU check-and-speed command line
// (sml/sml-gpu-fwd.c:2436-2660), on libsheep_b200.so.
//
//   sml-gpu-fwd MODEL.ssf ids,comma,separated NGEN
//
// Prints the lines the reference's tools parse (tooling/sml_tune.py:98-99
// RE_GPU / RE_GPU_GRADE; mlmi/backend/orchestrator.py parse_gpu_agreement):
//
//   GPU vs CPU over N positions: mean logit corr C, worst W, top-1 agree A/N
//   per-token path X tok/s (L launches per token)
//   GPU greedy decode: 64 tokens in S s = X tok/s, 1 launches/token, graph replay; tokens identical to the per-token path
//
// The reference links its CPU engine into this binary for the grade. This
// engine has no CPU path, so the grade reads the CPU engine's logits from a
// file instead: SML_CPU_LOGITS=FILE in the layout the reference's sml-cli
// writes with SML_ALL_LOGITS (int32 n_vocab and count, then count rows of
// n_vocab floats for positions 0..count-1 of the same ids, teacher-forced).
// Without it the grade line says that no comparison ran. The top-1 rule is the
// reference's: a different top token counts as agreeing when the CPU's two
// logits lie within 1 % of the CPU logits' standard deviation (a tie).
//
// Environment, as the reference reads it:
//   SML_LOGITS_OUT=FILE  read the ids through the prompt path and write the
//                        next-token logits (int32 n_vocab, 0, then the floats)
//   SML_PP=28,128,512    time the prompt path at these lengths (best of 3)
//   SPEED_ONLY           skip the grade
//   SML_CTX              context length (default 512)
#include "sheep_b200.h"
#include "sml-gpu.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double) ts.tv_sec + 1e-9 * (double) ts.tv_nsec;
}

static int argmax(const float * v, int n) {
    int a = 0;
    for (int i = 1; i < n; i++)
        if (v[i] > v[a]) a = i;
    return a;
}

// Pearson correlation of two logit vectors, the top tokens of each, and
// whether they agree (equal, or a tie within 1 % of the CPU logits' s.d.).
static double grade(const float * cpu, const float * gpu, int n, int * agree, int * tie) {
    double sa = 0, sb = 0, sab = 0, saa = 0, sbb = 0;
    for (int i = 0; i < n; i++) {
        const double a = cpu[i], b = gpu[i];
        sa += a; sb += b; sab += a * b; saa += a * a; sbb += b * b;
    }
    const double nn = n;
    const double corr = (sab - sa * sb / nn) / (sqrt((saa - sa * sa / nn) * (sbb - sb * sb / nn)) + 1e-30);
    const double sd = sqrt(saa / nn - (sa / nn) * (sa / nn));
    const int ac = argmax(cpu, n), ag = argmax(gpu, n);
    *tie = ac != ag && (double) cpu[ac] - (double) cpu[ag] <= 0.01 * sd;
    *agree = ac == ag || *tie;
    return corr;
}

int main(int argc, char ** argv) {
    if (argc < 4) { puts("usage: sml-gpu-fwd MODEL.ssf ids,comma,separated NGEN"); return 2; }
    const int ngen = atoi(argv[3]);
    int ids[512], nid = 0;
    for (char * s = argv[2]; *s && nid < 512;) {
        ids[nid++] = (int) strtol(s, &s, 10);
        while (*s == ',') s++;
    }
    if (nid < 1) { puts("  no ids"); return 2; }
    const int n_ctx = getenv("SML_CTX") ? atoi(getenv("SML_CTX")) : 512;
    char why[512];
    sb_engine * e = sb_open(argv[1], n_ctx, why, sizeof why);
    if (!e) { printf("  %s\n", why); return 1; }
    int info[13];
    sb_info(e, info);
    const int n_vocab = info[6], ctx = info[7];
    for (int i = 0; i < nid; i++)
        if (ids[i] < 0 || ids[i] >= n_vocab) { printf("  id %d out of range (vocab %d)\n", ids[i], n_vocab); return 1; }
    float * lg = (float *) malloc((size_t) n_vocab * sizeof(float));
    int rc = 0;

    if (getenv("SML_LOGITS_OUT")) {
        sb_set_prompt_mode(e, 2);
        const float * l = sb_prefill(e, ids, 0, nid);
        FILE * f = l ? fopen(getenv("SML_LOGITS_OUT"), "wb") : NULL;
        if (!f) {
            printf("  SML_LOGITS_OUT: %s\n", l ? "cannot open the file" : sb_last_error());
            rc = 1;
        } else {
            const int meta[2] = {n_vocab, 0};
            fwrite(meta, sizeof(int), 2, f);
            fwrite(l, sizeof(float), (size_t) n_vocab, f);
            fclose(f);
        }
        sb_close(e);
        free(lg);
        return rc;
    }

    if (getenv("SML_PP")) {
        sb_set_prompt_mode(e, 2);
        int * pid = (int *) malloc((size_t) ctx * sizeof(int));
        for (int i = 0; i < ctx; i++) pid[i] = i < nid ? ids[i] : (int) ((i * 7919u + 13u) % (unsigned) n_vocab);
        for (char * s = getenv("SML_PP"); *s;) {
            const int P = (int) strtol(s, &s, 10);
            while (*s == ',') s++;
            if (P <= 0 || P > ctx) { printf("  prompt %d skipped (n_ctx %d)\n", P, ctx); continue; }
            if (!sb_prefill(e, pid, 0, P)) { printf("  prompt %d: %s\n", P, sb_last_error()); rc = 1; break; }
            double best = 1e9;
            for (int rep = 0; rep < 3; rep++) {
                const double t0 = now_s();
                const float * l = sb_prefill(e, pid, 0, P);   // logits are copied to the host: synchronous
                const double dt = now_s() - t0;
                if (!l) { rc = 1; break; }
                if (dt < best) best = dt;
            }
            printf("  GPU prompt %4d tokens: %.1f ms = %.1f tok/s\n", P, best * 1e3, P / best);
        }
        free(pid);
        sb_close(e);
        free(lg);
        return rc;
    }

    // the grade: teacher-forced positions against the CPU engine's saved logits
    if (!getenv("SPEED_ONLY")) {
        const char * cpath = getenv("SML_CPU_LOGITS");
        FILE * f = cpath ? fopen(cpath, "rb") : NULL;
        int meta[2] = {0, 0};
        if (!f || fread(meta, sizeof(int), 2, f) != 2 || meta[0] != n_vocab || meta[1] < 1) {
            printf("  GPU vs CPU: %s\n", !cpath ? "no CPU logits (SML_CPU_LOGITS): no comparison ran"
                                                : "the CPU logits file does not match this model: no comparison ran");
        } else {
            const int npos = meta[1] < nid ? meta[1] : nid;
            float * lc = (float *) malloc((size_t) n_vocab * sizeof(float));
            double worst = 1.0, sumc = 0.0;
            int agree = 0, ties = 0, steps = 0;
            for (int pos = 0; pos < npos; pos++) {
                const float * l = sb_step(e, ids[pos], pos);
                if (!l || fread(lc, sizeof(float), (size_t) n_vocab, f) != (size_t) n_vocab) {
                    printf("  GPU vs CPU: %s\n", l ? "the CPU logits file is short" : sb_last_error());
                    rc = 1;
                    break;
                }
                int a = 0, t = 0;
                const double c = grade(lc, l, n_vocab, &a, &t);
                if (c < worst) worst = c;
                sumc += c;
                agree += a;
                ties += t;
                steps++;
            }
            if (steps == npos) {
                printf("  GPU vs CPU over %d positions: mean logit corr %.6f, worst %.6f, top-1 agree %d/%d", steps,
                       sumc / steps, worst, agree, steps);
                if (ties) printf(" (%d of them ties within 1%% of a logit s.d.)", ties);
                puts("");
            }
            free(lc);
        }
        if (f) fclose(f);
    }

    // speed: the per-token path (host ids in, host logits out, host argmax),
    // then the same tokens as graph replays with the choice on the device
    int nt = ngen > 0 ? ngen : 64;
    if (nt > 64) nt = 64;
    if (nt + 8 > ctx) nt = ctx - 8;
    int seq[64], dev[64];
    int tok = ids[0];
    for (int pos = 0; pos < 8 && rc == 0; pos++)
        if (!sb_step(e, tok, pos)) rc = 1;
    const double t0 = now_s();
    for (int pos = 0; pos < nt && rc == 0; pos++) {
        const float * l = sb_step(e, tok, pos);
        if (!l) { rc = 1; break; }
        tok = argmax(l, n_vocab);
        seq[pos] = tok;
    }
    const double tg = now_s() - t0;
    if (rc == 0) {
        printf("  per-token path %.2f tok/s (%d launches per token)\n", nt / tg, sb_launches_per_token(e));
        const double t1 = now_s();
        const int ok = sb_generate(e, ids, 1, nt, dev);
        const double tq = now_s() - t1;
        if (!ok) {
            printf("  GPU greedy decode: %s\n", sb_last_error());
            rc = 1;
        } else {
            const int same = memcmp(dev, seq, (size_t) nt * sizeof(int)) == 0;
            printf("  GPU greedy decode: %d tokens in %.2f s = %.2f tok/s, 1 launches/token, graph replay;"
                   " tokens %s the per-token path\n", nt, tq, nt / tq, same ? "identical to" : "DIFFER FROM");
        }
    } else {
        printf("  decode: %s\n", sb_last_error());
    }
    sb_close(e);
    free(lg);
    return rc;
}
