/* tcm-cuda: the reference's serving executable name (src/main.c dispatches
 * `serve` to src/qwen_serve.c), here over libcmachine_b200. Invoked as
 * tcm-bounded-chat it serves a byte-codec ring session. */
#include <stdio.h>
#include <string.h>

int qwen_serve_main(int argc, char **argv);

int main(int argc, char **argv) {
    if (argc >= 2 && !strcmp(argv[1], "serve")) return qwen_serve_main(argc, argv);
    fprintf(stderr, "usage: tcm-cuda serve MODEL [--context N] [--cache-policy native|full-byte|bounded]\n"
                    "MODEL: a TCM1LE bundle, or seeded:SHAPE:SEED:PROFILE\n");
    return 2;
}
