// g4sampler.hpp -- C++ host mirror of the reference's sampling surface, on top
// of the C ABI in g4sampler.h.
//
// The names follow the reference: TSamplingParams with SetDefaults
// (src/Gemma4.Model.pas:70-76, 346-352), and a sampler object whose DoSample
// takes the params record and returns the token id like
// TModel.DoSample (src/Gemma4.Model.pas:2739-2827).  Errors follow the
// reference's convention (src/Gemma4.Model.pas:57-59): methods return a Boolean
// or -1 and append a message to GetErrors(); nothing throws.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "g4sampler.h"

namespace g4 {

struct TSamplingParams : g4s_params {
    TSamplingParams() { SetDefaults(); }
    void SetDefaults() { g4s_params_defaults(this); }
};
static_assert(sizeof(TSamplingParams) == 16, "TSamplingParams must stay 16 bytes");

class TSampler {
public:
    TSampler() = default;
    TSampler(const TSampler &) = delete;
    TSampler &operator=(const TSampler &) = delete;
    ~TSampler() { Free(); }

    // Creates the device context (FConfig.VocabSize, FConfig.FinalLogitSoftcapping).
    bool Init(int32_t device, int32_t maxRows, int32_t vocabSize, float finalLogitSoftcapping,
              uint32_t flags = G4S_FLAG_HOST_STAGING)
    {
        Free();
        vocab_ = vocabSize;
        softcap_ = finalLogitSoftcapping;
        const int32_t rc = g4s_create(device, maxRows, vocabSize, flags, &ctx_);
        if (rc != G4S_OK) return AddError(rc, g4s_last_error(nullptr));
        return true;
    }

    void Free()
    {
        if (ctx_) g4s_destroy(ctx_);
        ctx_ = nullptr;
    }

    // DoSample on one host row of logits (FLogits) with draw u (the value of
    // Delphi's Random).  Returns the token id, or -1 with an error recorded.
    int32_t DoSample(const TSamplingParams &params, const float *hostLogits, double u)
    {
        if (!ctx_) {
            AddError(G4S_ERR_STATE, "TSampler.DoSample: Init was not called");
            return -1;
        }
        int32_t tok = -1;
        const int32_t rc = g4s_sample_host(ctx_, hostLogits, G4S_F32, 1, vocab_, vocab_, &params, 0,
                                           softcap_, &u, &tok);
        if (rc != G4S_OK) {
            AddError(rc, g4s_last_error(ctx_));
            return -1;
        }
        return tok;
    }

    // Batched device form: logits/u/outTokens are device pointers.
    bool SampleDevice(const void *logits, int32_t dtype, int32_t rows, int64_t rowStride,
                      const TSamplingParams *params, int32_t paramsStride, const double *u,
                      int32_t *outTokens, void *stream = nullptr)
    {
        if (!ctx_) return AddError(G4S_ERR_STATE, "TSampler.SampleDevice: Init was not called");
        const int32_t rc = g4s_sample(ctx_, logits, dtype, rows, vocab_, rowStride, params,
                                      paramsStride, softcap_, u, outTokens, stream);
        if (rc != G4S_OK) return AddError(rc, g4s_last_error(ctx_));
        return true;
    }

    const std::vector<std::string> &GetErrors() const { return errors_; }
    void ClearErrors() { errors_.clear(); }
    g4s_ctx *Handle() const { return ctx_; }

private:
    bool AddError(int32_t code, const char *msg)
    {
        errors_.push_back("G4S" + std::to_string(-code) + ": " + (msg ? msg : ""));
        return false;
    }

    g4s_ctx *ctx_ = nullptr;
    int32_t vocab_ = 0;
    float softcap_ = 0.0f;
    std::vector<std::string> errors_;
};

}  // namespace g4
