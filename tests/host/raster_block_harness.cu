// Host run of the raster forward's splat-versus-block tests (the
// __host__ __device__ pack_record, block_hit and ellipse_hit of
// jaxgs_b200/csrc/raster.cu) on splats given as (mean, conic, opacity),
// against the pixel-centre rectangles of an 8 x 4 (ROWS = 1) and an 8 x 8
// (ROWS = 2) block at the origin.  Test infrastructure: the product runs
// these functions on the GPU only.
//
// usage: raster_block_harness splats.f32 out.u8
// splats.f32: N x 7 floats (mean_x, mean_y, c00, c01, c10, c11, opacity);
// out.u8: N x 4 flags (bbox ROWS=1, bbox+ellipse ROWS=1, bbox ROWS=2,
// bbox+ellipse ROWS=2).
#include "../../jaxgs_b200/csrc/raster.cu"

#include <cstdio>
#include <vector>

namespace gsb {
void set_error(cudaError_t) {}
void set_error_text(const char*) {}
void count_launch() {}
}  // namespace gsb

using namespace gsb;

int main(int argc, char** argv)
{
    if (argc != 3) return 2;
    FILE* f = fopen(argv[1], "rb");
    if (!f) return 3;
    std::vector<float> in;
    float v[7];
    while (fread(v, sizeof(float), 7, f) == 7) in.insert(in.end(), v, v + 7);
    fclose(f);
    const size_t n = in.size() / 7;
    std::vector<unsigned char> out(n * 4);
    for (size_t i = 0; i < n; i++) {
        const float* s = &in[i * 7];
        float4 r[3];
        pack_record(make_float2(s[0], s[1]), make_float4(s[2], s[3], s[4], s[5]), s[6], 0.5f, 0.5f,
                    0.5f, r);
        const bool b1 = block_hit<1>(r[0], 0.0f, 0.0f), b2 = block_hit<2>(r[0], 0.0f, 0.0f);
        out[i * 4 + 0] = b1;
        out[i * 4 + 1] = b1 && ellipse_hit<1>(r[0], r[1], r[2].w, 0.0f, 0.0f);
        out[i * 4 + 2] = b2;
        out[i * 4 + 3] = b2 && ellipse_hit<2>(r[0], r[1], r[2].w, 0.0f, 0.0f);
    }
    FILE* o = fopen(argv[2], "wb");
    if (!o) return 4;
    fwrite(out.data(), 1, out.size(), o);
    fclose(o);
    return 0;
}
