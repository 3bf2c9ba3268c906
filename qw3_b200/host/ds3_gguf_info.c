/*
 * ds3_gguf_info - open a GGUF file through include/ds3_cuda_gguf.h, print its
 * header and tensor table, check that every tensor lies inside the file, and
 * (with -b) bind the fused path's tensors to device buffers.
 *
 * Plays the role of the engine's tests/test_gguf.c (parse + summary, data
 * pointers inside the mapping, optional binding) for this backend:
 *
 *   ds3_gguf_info model.gguf            header + table (no GPU needed)
 *   ds3_gguf_info model.gguf -b N       also bind N layers on the GPU
 *
 * Output lines (one per item, space separated) are meant for scripts:
 *   header <version> <alignment> <n_tensors> <n_metadata> <data_offset>
 *   tensor <name> <n_dims> <ne0> <ne1> <ne2> <ne3> <type> <offset> <size>
 *   bound <n_layer> <n_embd> <n_vocab> <head_dim> <n_expert> <embd_type>
 * Exit codes: 0 ok, 1 parse or bind failure, 77 when -b is asked for and no
 * GPU is usable (the reference tests' skip code).
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "ds3_cuda_gguf.h"

int main(int argc, char **argv)
{
    if (argc < 2) {
        fprintf(stderr, "usage: %s FILE.gguf [-b N_LAYER]\n", argv[0]);
        return 1;
    }
    int bind_layers = 0;
    for (int i = 2; i + 1 < argc; i++)
        if (strcmp(argv[i], "-b") == 0) bind_layers = atoi(argv[i + 1]);

    ds3_cuda_gguf_t *g = ds3_cuda_gguf_open(argv[1]);
    if (!g) {
        fprintf(stderr, "open failed: %s\n", ds3_cuda_last_error());
        return 1;
    }
    const uint64_t n = ds3_cuda_gguf_n_tensors(g);
    printf("header %u %u %llu %llu %llu\n", ds3_cuda_gguf_version(g), ds3_cuda_gguf_alignment(g),
           (unsigned long long)n, (unsigned long long)ds3_cuda_gguf_n_metadata(g),
           (unsigned long long)ds3_cuda_gguf_data_offset(g));
    uint64_t total = 0;
    for (uint64_t i = 0; i < n; i++) {
        ds3_cuda_gguf_tensor_t t;
        if (ds3_cuda_gguf_tensor(g, i, &t) != 0) {
            ds3_cuda_gguf_close(g);
            return 1;
        }
        printf("tensor %.*s %u %llu %llu %llu %llu %u %llu %llu\n", (int)t.name_len, t.name, t.n_dims,
               (unsigned long long)t.ne[0], (unsigned long long)t.ne[1], (unsigned long long)t.ne[2],
               (unsigned long long)t.ne[3], t.type, (unsigned long long)t.offset, (unsigned long long)t.size);
        total += t.size;
    }
    fprintf(stderr, "%llu tensors, %llu bytes of tensor data, all inside the file\n", (unsigned long long)n,
            (unsigned long long)total);

    int rc = 0;
    if (bind_layers > 0) {
        if (ds3_cuda_init() != 0) {
            fprintf(stderr, "no usable GPU: %s\n", ds3_cuda_last_error());
            ds3_cuda_gguf_close(g);
            return 77;
        }
        ds3_cuda_path_weights_t *w = ds3_cuda_path_weights_load(g, (uint32_t)bind_layers, true);
        if (!w) {
            fprintf(stderr, "bind failed: %s\n", ds3_cuda_last_error());
            rc = 1;
        } else {
            printf("bound %u %u %u %u %u %u\n", w->n_layer, w->n_embd, w->n_vocab, w->head_dim, w->n_expert,
                   w->token_embd_type);
            ds3_cuda_path_weights_free(w);
        }
        ds3_cuda_shutdown();
    }
    ds3_cuda_gguf_close(g);
    return rc;
}
