/* Driver for a generated C wrapper (symbol `model`, see
 * spinnv2_b200/compiler/c_codegen.py): reads the package's inputs, one after
 * the other, from argv[1]; runs the model `runs` times (argv[3], default 2)
 * through model_run (one input, one output) or model_run_multi (otherwise);
 * writes the outputs of the last run, one after the other, to argv[2].
 * Exit code: 0 on success, else 100 + |runtime code| (file errors 2). */
#include <stdio.h>
#include <stdlib.h>

#include "model.h"

int main(int argc, char **argv) {
    if (argc < 3) return 2;
    int runs = argc > 3 ? atoi(argv[3]) : 2;
    size_t in_sizes[] = MODEL_INPUT_SIZES, out_sizes[] = MODEL_OUTPUT_SIZES;
    const void *ins[MODEL_INPUT_COUNT];
    void *outs[MODEL_OUTPUT_COUNT];
    FILE *f = fopen(argv[1], "rb");
    if (!f) return 2;
    for (int i = 0; i < MODEL_INPUT_COUNT; ++i) {
        void *b = malloc(in_sizes[i]);
        if (!b || fread(b, 1, in_sizes[i], f) != in_sizes[i]) return 2;
        ins[i] = b;
    }
    fclose(f);
    for (int i = 0; i < MODEL_OUTPUT_COUNT; ++i)
        if (!(outs[i] = malloc(out_sizes[i]))) return 2;
    if (model_verify_checksum(ins[0], 0) != -1) return 3; /* empty buffer is a bad argument */
    for (int r = 0; r < runs; ++r) {
        int rc = (MODEL_INPUT_COUNT == 1 && MODEL_OUTPUT_COUNT == 1)
                     ? model_run(ins[0], outs[0])
                     : model_run_multi(ins, in_sizes, MODEL_INPUT_COUNT, outs, out_sizes, MODEL_OUTPUT_COUNT);
        if (rc != 0) {
            fprintf(stderr, "model run failed: %d\n", rc);
            return 100 + (rc < 0 ? -rc : rc) % 100;
        }
    }
    if (model_run_checked(ins[0], MODEL_INPUT_SIZE + 1, outs[0], MODEL_OUTPUT_SIZE) != -2) return 4;
    f = fopen(argv[2], "wb");
    if (!f) return 2;
    for (int i = 0; i < MODEL_OUTPUT_COUNT; ++i)
        if (fwrite(outs[i], 1, out_sizes[i], f) != out_sizes[i]) return 2;
    fclose(f);
    model_free();
    return 0;
}
