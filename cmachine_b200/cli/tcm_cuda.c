/* tcm-cuda: the reference's executable names over libcmachine_b200 (src/main.c
 * dispatches `qwen` to the timed run and `serve` to the line protocol). Invoked
 * as tcm-bounded-chat it serves a byte-codec ring session. */
#include <stdio.h>
#include <string.h>

int qwen_main(int argc, char **argv);
int qwen_serve_main(int argc, char **argv);

int main(int argc, char **argv) {
    if (argc >= 2 && !strcmp(argv[1], "qwen")) return qwen_main(argc, argv);
    if (argc >= 2 && !strcmp(argv[1], "serve")) return qwen_serve_main(argc, argv);
    fprintf(stderr, "usage: tcm-cuda qwen MODEL --tokens-file F [--new-tokens N] [--context C] [--output P]\n"
                    "         [--first-logits P] [--checkpoint-test] [--trace-prefix P --trace-layer L [--trace-position T]]\n"
                    "       tcm-cuda serve MODEL [--context N] [--cache-policy native|full-byte|bounded]\n"
                    "MODEL: a TCM1LE bundle, or seeded:SHAPE:SEED:PROFILE\n");
    return 2;
}
