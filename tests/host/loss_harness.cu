// Host run of the fused loss kernel's stage and pass bodies (the
// __host__ __device__ functions of jaxgs_b200/csrc/loss.cu), thread by
// thread between the kernel's barriers, every CTA of the launch grid in
// turn, with the shared state filled with NaN before each CTA so that a
// read of a row the kernel never staged poisons the output.  Built with
// -fsanitize=bounds so that every shared-memory index is range-checked.
// Test infrastructure: the product runs these bodies on the GPU only.
//
// usage: loss_harness W H u8 clip image.f32 target(.u8|.f32) grad.f32 out.f32
// out.f32 = (loss, max |grad|, rows per segment, CTAs).
#include "../../jaxgs_b200/csrc/loss.cu"

#include <cstdlib>
#include <limits>
#include <vector>

namespace gsb {
void set_error(cudaError_t) {}
void set_error_text(const char*) {}
void count_launch() {}
}  // namespace gsb

using namespace gsb;

template <bool U8, bool CLIP>
static void run(int W, int H, const float* image, const void* target, float* grad, float* out)
{
    gsb_loss_params p{W, H, U8, CLIP};
    const int seg_rows = loss_segment_rows(p);
    const int strips = ceil_div(W, kTW), segs = ceil_div(H, seg_rows);
    std::vector<float> block_loss;
    std::vector<uint32_t> block_scale;
    LossSmem* S = new LossSmem;
    for (int c = 0; c < 3; c++)
        for (int by = 0; by < segs; by++)
            for (int bx = 0; bx < strips; bx++) {
                float* raw = reinterpret_cast<float*>(S);
                for (size_t i = 0; i < sizeof(LossSmem) / sizeof(float); i++)
                    raw[i] = std::numeric_limits<float>::quiet_NaN();
                const Strip g = strip_of(W, H, seg_rows, bx, by, c);
                float loss[kThreads] = {};
                uint32_t scale[kThreads] = {};
                for (int k = 0; k < strip_chunks(g); k++) {
                    if (k == 0)
                        for (int t = 0; t < kThreads; t++) stage_rows<U8, CLIP>(t, *S, g, 0, image, target);
                    for (int t = 0; t < kThreads; t++) stage_rows<U8, CLIP>(t, *S, g, k + 1, image, target);
                    for (int t = 0; t < kThreads; t++) pass1(t, *S, g, k);
                    for (int t = 0; t < kThreads; t++) pass2(t, *S, g, k, loss[t]);
                    if (k > 0) {
                        for (int t = 0; t < kThreads; t++) pass3(t, *S, g, k);
                        for (int t = 0; t < kThreads; t++)
                            pass4<CLIP>(t, *S, g, k, image, grad, loss[t], scale[t]);
                    }
                }
                float total = 0.0f;
                uint32_t sb = 0;
                for (int t = 0; t < kThreads; t++) {
                    total += loss[t];
                    sb = sb > scale[t] ? sb : scale[t];
                }
                block_loss.push_back(total);
                block_scale.push_back(sb);
            }
    delete S;
    double sum = 0.0;
    uint32_t m = 0;
    for (size_t i = 0; i < block_loss.size(); i++) {
        sum += block_loss[i];
        m = m > block_scale[i] ? m : block_scale[i];
    }
    out[0] = (float)(sum * (double)(1.0f / (3.0f * (float)W * (float)H)));
    std::memcpy(&out[1], &m, sizeof(float));
    out[2] = (float)seg_rows;
    out[3] = (float)block_loss.size();
}

static std::vector<char> slurp(const char* path)
{
    FILE* f = std::fopen(path, "rb");
    if (!f) std::abort();
    std::fseek(f, 0, SEEK_END);
    const long n = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    std::vector<char> bytes(n);
    if (std::fread(bytes.data(), 1, n, f) != (size_t)n) std::abort();
    std::fclose(f);
    return bytes;
}

int main(int argc, char** argv)
{
    if (argc != 9) return 2;
    const int W = std::atoi(argv[1]), H = std::atoi(argv[2]);
    const bool u8 = std::atoi(argv[3]) != 0, clip = std::atoi(argv[4]) != 0;
    const std::vector<char> img = slurp(argv[5]), tgt = slurp(argv[6]);
    std::vector<float> grad((size_t)W * H * 3, std::numeric_limits<float>::quiet_NaN());
    float out[4];
    const float* im = reinterpret_cast<const float*>(img.data());
    if (u8) {
        if (clip) run<true, true>(W, H, im, tgt.data(), grad.data(), out);
        else run<true, false>(W, H, im, tgt.data(), grad.data(), out);
    } else {
        if (clip) run<false, true>(W, H, im, tgt.data(), grad.data(), out);
        else run<false, false>(W, H, im, tgt.data(), grad.data(), out);
    }
    FILE* f = std::fopen(argv[7], "wb");
    std::fwrite(grad.data(), sizeof(float), grad.size(), f);
    std::fclose(f);
    f = std::fopen(argv[8], "wb");
    std::fwrite(out, sizeof(float), 4, f);
    std::fclose(f);
    return 0;
}
