// Test infrastructure (not product code): a host-only cuBLASLt query behind the record of why the reference's
// effort-1 GEMM tuning cannot run on B200. For every algorithm id of the reference's GEMM types (fp16 A/B, fp32
// compute, fp16 or fp32 C/D; cuda/gemm.cu:59-75) it prints how many tile ids the CUBLASLT_ALGO_CAP_TILE_IDS
// attribute holds. cuda/gemm.cu:198-203 reads that attribute into a fixed `int tiles[128]` stack array; an algorithm
// listing more than 128 tiles overruns it. No matmul runs and no GPU kernel is launched.
//   make -C oracle probe && oracle/_ref/cublaslt_tiles
#include <cublasLt.h>
#include <cuda_runtime.h>
#include <stdio.h>
int main() {
    cublasLtHandle_t lt;
    if (cublasLtCreate(&lt)) { printf("create failed\n"); return 1; }
    printf("cublasLt %zu\n", cublasLtGetVersion());
    for (int yf32 = 0; yf32 < 2; yf32++) {
        cudaDataType_t yt = yf32 ? CUDA_R_32F : CUDA_R_16F;
        int ids[1024], nid = 0;
        cublasLtMatmulAlgoGetIds(lt, CUBLAS_COMPUTE_32F, CUDA_R_32F, CUDA_R_16F, CUDA_R_16F, yt, yt, 1024, ids, &nid);
        int over = 0, maxnt = 0;
        for (int a = 0; a < nid; a++) {
            cublasLtMatmulAlgo_t algo;
            if (cublasLtMatmulAlgoInit(lt, CUBLAS_COMPUTE_32F, CUDA_R_32F, CUDA_R_16F, CUDA_R_16F, yt, yt, ids[a], &algo)) continue;
            size_t sz = 0;
            cublasLtMatmulAlgoCapGetAttribute(&algo, CUBLASLT_ALGO_CAP_TILE_IDS, nullptr, 0, &sz);
            int nt = (int)(sz / sizeof(int));
            if (nt > maxnt) maxnt = nt;
            if (nt > 128) over++;
            printf("y_f32=%d algo_id=%d tiles=%d\n", yf32, ids[a], nt);
        }
        printf("y_f32=%d: %d algorithm ids (request 1024), max tiles %d, %d with more than 128 tiles\n", yf32, nid, maxnt, over);
    }
    cublasLtDestroy(lt);
    return 0;
}
