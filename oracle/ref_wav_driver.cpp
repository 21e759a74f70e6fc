// Oracle driver for the reference CLI's WAV reader.
//
// Test infrastructure only: built by oracle/Makefile into oracle/_ref/ from
// the reference checkout.  The reader, load_wav (examples/main/main.cpp:20-82),
// is file-static in the CLI source, so that source is compiled into this
// translation unit unmodified (its main() renamed by the preprocessor) and
// the reader is exported through one C entry point.  The CLI's calls into the
// wav2vec2 API resolve to the reference build linked beside it.
#define main w2vref_cli_main
#include "main.cpp"   // reference examples/main/main.cpp (found via -I<ref>/examples/main)
#undef main

extern "C" {

// Decode path at target_sr into out (capacity cap floats).  Returns the
// sample count, or -1 with the reference's exception message in err, or -2
// if cap is too small.
long w2vref_load_wav(const char * path, int target_sr, float * out, long cap, char * err, int err_cap) {
    try {
        std::vector<float> a = load_wav(path, target_sr);
        if ((long)a.size() > cap) return -2;
        if (!a.empty()) memcpy(out, a.data(), a.size() * sizeof(float));
        return (long)a.size();
    } catch (const std::exception & e) {
        snprintf(err, (size_t)err_cap, "%s", e.what());
        return -1;
    }
}

}
