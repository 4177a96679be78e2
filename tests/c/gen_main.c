/* Driver for a generated C wrapper (symbol `model`, see
 * spinnv2_b200/compiler/c_codegen.py): reads MODEL_INPUT_SIZE bytes from
 * argv[1], calls model_run `runs` times (argv[3], default 2), writes
 * MODEL_OUTPUT_SIZE bytes of the last run to argv[2].  Exit code: 0 on
 * success, else 100 + |runtime code| (file errors 2). */
#include <stdio.h>
#include <stdlib.h>

#include "model.h"

int main(int argc, char **argv) {
    if (argc < 3) return 2;
    int runs = argc > 3 ? atoi(argv[3]) : 2;
    unsigned char *in = malloc(MODEL_INPUT_SIZE), *out = malloc(MODEL_OUTPUT_SIZE);
    if (!in || !out) return 2;
    FILE *f = fopen(argv[1], "rb");
    if (!f || fread(in, 1, MODEL_INPUT_SIZE, f) != MODEL_INPUT_SIZE) return 2;
    fclose(f);
    if (model_verify_checksum(in, 0) != -1) return 3; /* empty buffer is a bad argument */
    for (int i = 0; i < runs; ++i) {
        int rc = model_run(in, out);
        if (rc != 0) {
            fprintf(stderr, "model_run failed: %d\n", rc);
            return 100 + (rc < 0 ? -rc : rc) % 100;
        }
    }
    if (model_run_checked(in, MODEL_INPUT_SIZE + 1, out, MODEL_OUTPUT_SIZE) != -2) return 4;
    f = fopen(argv[2], "wb");
    if (!f || fwrite(out, 1, MODEL_OUTPUT_SIZE, f) != MODEL_OUTPUT_SIZE) return 2;
    fclose(f);
    model_free();
    free(in);
    free(out);
    return 0;
}
