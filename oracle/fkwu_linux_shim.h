/* fkwu_linux_shim.h -- force-included when the reference runtime (runtime/fkwu-uni.c) is compiled
 * on Linux.  That file uses two names that it defines only inside its Darwin/arm64 JIT block
 * (fk_melt_gen and fk_jit_leaf_inram); these are the inert definitions the Linux build lacks.
 * Nothing else about the reference file is changed. */
static long long fk_melt_gen = 0;
static long long fk_jit_leaf_inram(long long a, long long b) { (void)a; (void)b; return 0; }
