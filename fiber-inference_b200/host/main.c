/* main.c — fiber-inference command-line driver (GGUF decode on one B200).
 *
 * Same flags, defaults and output as the reference CLI's GGUF path
 * (src/main.m:27-40, 356-612): --model --prompt --tokens --ctx-len
 * --temperature --top-k --top-p --list-tensors --benchmark --help, prompt
 * prefilled token by token, generated text streamed, then the "--- Stats ---"
 * block with Prefill/Decode tok/s. With --temperature <= 0 the greedy argmax is
 * taken on the device and the logits never leave HBM; otherwise the logits are
 * copied back and sampled by the host sampler (top-k / top-p).
 * Additions: --gpu N (device ordinal), --synth PRESET (write a seeded synthetic
 * model to --model's path first: stories, tinyllama, tinyllama-q5, llama7b),
 * --ids (also print the prompt and generated token ids to stderr). The prompt is
 * prefilled with one fiber_prefill call (batched on the tensor cores) instead of
 * the reference's token-by-token loop.
 * --no-ane and --arch belong to Apple-only paths and are not accepted.
 */
#include <getopt.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "fiber_cuda.h"
#include "fiber_synth.h"
#include "model.h"
#include "fiber_ckpt.h"
#include "sampler.h"
#include "tokenizer.h"

#define MAX_PROMPT_TOKENS 4096

static double now_ms(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec * 1e3 + t.tv_nsec / 1e6;
}

static void usage(const char *prog) {
    fprintf(stderr, "Usage: %s --model <path.gguf> [options]\n", prog);
    fprintf(stderr, "\nOptions:\n");
    fprintf(stderr, "  --model <path>      Path to GGUF model file (required); a karpathy/llama2.c .bin\n");
    fprintf(stderr, "                      checkpoint is rewritten as a GGUF in $TMPDIR (or /tmp) first\n");
    fprintf(stderr, "  --prompt <text>     Input prompt (default: \"Hello\")\n");
    fprintf(stderr, "  --tokens <n>        Max tokens to generate (default: 128)\n");
    fprintf(stderr, "  --ctx-len <n>       Max context length (default: model max)\n");
    fprintf(stderr, "  --temperature <f>   Sampling temperature (default: 0.7; <= 0 is greedy on the GPU)\n");
    fprintf(stderr, "  --top-k <n>         Top-k sampling (default: 40)\n");
    fprintf(stderr, "  --top-p <f>         Top-p (nucleus) sampling (default: 0.9)\n");
    fprintf(stderr, "  --list-tensors      List all tensors and exit\n");
    fprintf(stderr, "  --benchmark         Print per-token timing\n");
    fprintf(stderr, "  --gpu <n>           CUDA device ordinal (default: 0)\n");
    fprintf(stderr, "  --synth <preset>    Write a seeded synthetic model to --model first\n");
    fprintf(stderr, "  --ids               Also print prompt and generated token ids to stderr\n");
    fprintf(stderr, "  --help              Show this help\n");
}

static void list_tensors(const model_t *m) {
    printf("\n=== Tensor Index (%llu tensors) ===\n", (unsigned long long)m->gf->n_tensors);
    for (uint64_t i = 0; i < m->gf->n_tensors; i++) {
        const gguf_tensor_info_t *ti = &m->gf->tensors[i];
        char shape[64];
        if (ti->n_dims == 1)
            snprintf(shape, sizeof(shape), "[%llu]", (unsigned long long)ti->dims[0]);
        else
            snprintf(shape, sizeof(shape), "[%llu, %llu]", (unsigned long long)ti->dims[0],
                     (unsigned long long)ti->dims[1]);
        int n = (int)(ti->name.len < 50 ? ti->name.len : 50);
        printf("  %-45.*s %-6s %s\n", n, ti->name.str, ggml_type_name(ti->type), shape);
    }
}

int main(int argc, char **argv) {
    const char *model_path = NULL, *prompt = "Hello", *synth = NULL;
    int max_gen = 128, top_k = 40, list_flag = 0, bench_flag = 0, device = 0, ids_flag = 0;
    unsigned ctx_len = 0;
    float temperature = 0.7f, top_p = 0.9f;
    static struct option opts[] = {
        {"model", required_argument, 0, 'm'},       {"prompt", required_argument, 0, 'p'},
        {"tokens", required_argument, 0, 'n'},      {"ctx-len", required_argument, 0, 'c'},
        {"temperature", required_argument, 0, 'T'}, {"top-k", required_argument, 0, 'k'},
        {"top-p", required_argument, 0, 'P'},       {"list-tensors", no_argument, 0, 't'},
        {"benchmark", no_argument, 0, 'b'},         {"gpu", required_argument, 0, 'g'},
        {"synth", required_argument, 0, 's'},       {"help", no_argument, 0, 'h'},
        {"ids", no_argument, 0, 'i'},               {0, 0, 0, 0}};
    int o;
    while ((o = getopt_long(argc, argv, "m:p:n:c:T:k:P:tbh", opts, NULL)) != -1) {
        switch (o) {
        case 'm': model_path = optarg; break;
        case 'p': prompt = optarg; break;
        case 'n': max_gen = atoi(optarg); break;
        case 'c': ctx_len = (unsigned)atoi(optarg); break;
        case 'T': temperature = (float)atof(optarg); break;
        case 'k': top_k = atoi(optarg); break;
        case 'P': top_p = (float)atof(optarg); break;
        case 't': list_flag = 1; break;
        case 'b': bench_flag = 1; break;
        case 'g': device = atoi(optarg); break;
        case 's': synth = optarg; break;
        case 'i': ids_flag = 1; break;
        case 'h': usage(argv[0]); return 0;
        default: usage(argv[0]); return 1;
        }
    }
    if (!model_path) {
        fprintf(stderr, "Error: --model is required\n");
        usage(argv[0]);
        return 1;
    }
    if (synth) {
        fiber_synth_cfg_t cfg;
        if (fiber_synth_preset(synth, &cfg) != 0) {
            fprintf(stderr, "Error: unknown --synth preset %s\n", synth);
            return 1;
        }
        printf("Writing synthetic %s model to %s\n", synth, model_path);
        if (fiber_synth_write_gguf(model_path, &cfg) != 0) return 1;
    }

    printf("Fiber-Inference B200 (CUDA decode path)\n\n");
    printf("Loading: %s\n", model_path);
    double t0 = now_ms();
    model_t *m = NULL;
    const size_t plen = strlen(model_path);
    if (plen > 4 && strcmp(model_path + plen - 4, ".bin") == 0) {
        const char *dir = getenv("TMPDIR");
        const char *base = strrchr(model_path, '/');
        char gguf_path[4096];
        snprintf(gguf_path, sizeof(gguf_path), "%s/%s.gguf", dir && *dir ? dir : "/tmp", base ? base + 1 : model_path);
        printf("karpathy checkpoint: writing %s\n", gguf_path);
        m = model_open_karpathy(model_path, gguf_path);
    } else {
        m = model_open(model_path);
    }
    if (!m) {
        fprintf(stderr, "Failed to open model\n");
        return 1;
    }
    printf("Model loaded in %.1f ms\n\n", now_ms() - t0);
    model_print_info(m);
    if (list_flag) {
        list_tensors(m);
        model_close(m);
        return 0;
    }
    if (ctx_len == 0 || ctx_len > m->params.context_length) ctx_len = m->params.context_length;

    t0 = now_ms();
    tokenizer_t *tok = tokenizer_init(m->gf);
    if (!tok) {
        fprintf(stderr, "Failed to init tokenizer\n");
        model_close(m);
        return 1;
    }
    printf("Tokenizer initialized in %.1f ms\n", now_ms() - t0);

    t0 = now_ms();
    fiber_ctx_t *gpu = fiber_cuda_init(m, device, 1, (int)ctx_len);
    if (!gpu) {
        fprintf(stderr, "Failed to init GPU: %s\n", fiber_last_error());
        tokenizer_free(tok);
        model_close(m);
        return 1;
    }
    printf("GPU initialized in %.1f ms\n", now_ms() - t0);
    kv_cache_t *kv = kv_cache_init(device, (int)m->params.n_layers, (int)m->params.n_kv_heads,
                                   (int)m->params.head_dim, (int)ctx_len);
    if (!kv) {
        fprintf(stderr, "Failed to init KV cache: %s\n", fiber_last_error());
        fiber_cuda_free(gpu);
        tokenizer_free(tok);
        model_close(m);
        return 1;
    }
    sampler_t sampler;
    sampler_init(&sampler, (int)m->params.vocab_size, temperature, top_k, top_p);
    const int greedy = temperature <= 0.0f || temperature < 1e-6f;
    float *logits = greedy ? NULL : (float *)malloc(m->params.vocab_size * sizeof(float));

    static int prompt_tokens[MAX_PROMPT_TOKENS];
    int n_prompt = tokenizer_encode(tok, prompt, prompt_tokens, MAX_PROMPT_TOKENS);
    if (n_prompt == 0) {
        prompt_tokens[0] = tokenizer_bos(tok);
        n_prompt = 1;
    }
    if (n_prompt >= (int)ctx_len) n_prompt = (int)ctx_len - 1;
    printf("\nPrompt: \"%s\" → %d tokens\n", prompt, n_prompt);
    printf("RSS after init: %.1f MB\n", model_get_rss() / (1024.0 * 1024.0));
    printf("\n--- Output ---\n");
    for (int i = 0; i < n_prompt; i++) printf("%s", tokenizer_decode(tok, prompt_tokens[i]));
    fflush(stdout);

    if (ids_flag) {
        fprintf(stderr, "prompt ids:");
        for (int i = 0; i < n_prompt; i++) fprintf(stderr, " %d", prompt_tokens[i]);
        fprintf(stderr, "\n");
    }

    // prefill: the whole prompt in one call (greedy), or all but the last token and
    // then the last one with its logits for the sampler
    int rc = 0, next = 0;
    t0 = now_ms();
    {
        int32_t am = 0;
        const int n_pre = greedy ? n_prompt : n_prompt - 1;
        if (n_pre > 0) rc = fiber_prefill(gpu, kv, prompt_tokens, n_pre, 0, &am);
        if (rc == 0 && !greedy) {
            const int32_t tk = prompt_tokens[n_prompt - 1], ps = n_prompt - 1;
            rc = fiber_forward_token(gpu, kv, &tk, &ps, 1, logits, &am);
        }
        next = am;
    }
    const double prefill_ms = now_ms() - t0;
    if (rc == 0 && !greedy) next = sampler_sample(&sampler, logits);
    int *gen_ids = ids_flag ? (int *)malloc((size_t)(max_gen > 0 ? max_gen : 1) * sizeof(int)) : NULL;

    int pos = n_prompt, gen = 0;
    const double g0 = now_ms();
    for (int i = 0; rc == 0 && i < max_gen && pos < (int)ctx_len; i++) {
        printf("%s", tokenizer_decode(tok, next));
        fflush(stdout);
        if (gen_ids) gen_ids[gen] = next;
        gen++;
        if (next == tokenizer_eos(tok)) break;
        const double s0 = now_ms();
        const int32_t tk = next, ps = pos;
        int32_t am = 0;
        rc = fiber_forward_token(gpu, kv, &tk, &ps, 1, greedy ? NULL : logits, &am);
        next = greedy ? am : sampler_sample(&sampler, logits);
        if (bench_flag) fprintf(stderr, "[token %d] %.3f ms\n", i, now_ms() - s0);
        pos++;
    }
    const double gen_ms = now_ms() - g0;
    if (rc != 0) fprintf(stderr, "\nError: %s\n", fiber_last_error());
    if (gen_ids) {
        fprintf(stderr, "generated ids:");
        for (int i = 0; i < gen; i++) fprintf(stderr, " %d", gen_ids[i]);
        fprintf(stderr, "\n");
        free(gen_ids);
    }

    printf("\n\n--- Stats ---\n");
    printf("Prefill: %d tokens in %.1f ms (%.1f tok/s)\n", n_prompt, prefill_ms, n_prompt / (prefill_ms / 1000.0));
    if (gen > 0) printf("Decode:  %d tokens in %.1f ms (%.1f tok/s)\n", gen, gen_ms, gen / (gen_ms / 1000.0));
    printf("Peak RSS: %.1f MB\n", model_get_rss() / (1024.0 * 1024.0));

    free(logits);
    kv_cache_free(kv);
    fiber_cuda_free(gpu);
    tokenizer_free(tok);
    model_close(m);
    return rc == 0 ? 0 : 1;
}
