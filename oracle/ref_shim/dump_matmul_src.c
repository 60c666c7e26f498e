/* dump_matmul_src.c -- write the matmul kernel source that the reference's
 * build_matmul_kernel (main.c:686-716) generates for one tile shape.
 *
 * TEST INFRASTRUCTURE ONLY.  A build-time tool of oracle/Makefile: it includes
 * the reference's main.c (main renamed on the compile line) to reach its
 * MATMUL_SRC_FMT template and prints it for tile 64x64x16 / 4x4, so that the
 * generated kernel can be compiled ahead of time for the CPU OpenCL shim.
 */
#include "main.c"
#undef main

int main(int argc, char **argv) {
    if (argc != 2) return 2;
    FILE *f = fopen(argv[1], "w");
    if (!f) return 1;
    fprintf(f, MATMUL_SRC_FMT, 64, 64, 16, 4, 4);
    return fclose(f) == 0 ? 0 : 1;
}
