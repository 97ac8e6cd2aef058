unit G4Sampler;

{ Object Pascal binding of libg4sampler.so -- the B200 token sampler that
  replaces TModel.DoSample (src/Gemma4.Model.pas:2739-2827 of Gemma4.pas).

  Mirrors include/g4sampler.h one to one: cdecl entry points, plain pointers
  and sizes, Int32 status results (G4S_OK = 0, negative on error) and a
  per-context error text (g4s_last_error), in the same spirit as the
  reference's Boolean results plus GetErrors().

  Targets Free Pascal ({$MODE DELPHI}) and Delphi for Linux64.  It does not
  include StdApp.Defines.inc, which rejects non-Win64 targets
  (src/vendor/StdApp/StdApp.Defines.inc:33-35). }

{$IFDEF FPC}{$MODE DELPHI}{$ENDIF}

interface

const
  G4SLib = 'libg4sampler.so';

  G4S_ABI_VERSION = 2;

  G4S_OK              = 0;
  G4S_ERR_ARG         = -1;
  G4S_ERR_CUDA        = -2;
  G4S_ERR_NOMEM       = -3;
  G4S_ERR_CAPACITY    = -4;
  G4S_ERR_NCCL        = -5;
  G4S_ERR_TIMEOUT     = -6;
  G4S_ERR_STATE       = -7;
  G4S_ERR_UNAVAILABLE = -8;

  G4S_F32  = 0;
  G4S_BF16 = 1;

  G4S_FLAG_HOST_STAGING = 1;

  G4S_ROW_FALLBACK  = 1;
  G4S_ROW_EMPTY     = 2;
  G4S_ROW_FULL_PATH = 4;
  G4S_ROW_GREEDY    = 8;

  G4S_PHASE_FULL_STREAM_ONLY = 1;
  G4S_PHASE_LMHEAD_UNFUSED = 2;

  G4S_NOALLOC_MAX_ROWS  = 64;
  G4S_NOALLOC_MAX_LISTS = 1024;

  G4S_SHARD_LIST      = 256;   { composites per row per shard list }
  G4S_SHARD_UID_BYTES = 128;

type
  { Same layout as TSamplingParams (src/Gemma4.Model.pas:70-76): four 4-byte
    fields at offsets 0/4/8/12, so a TSamplingParams can be passed by address. }
  TG4SParams = record
    Temperature: Single;
    TopK: Int32;
    TopP: Single;
    RepetitionPenalty: Single;
  end;
  PG4SParams = ^TG4SParams;

  TG4SOutputs = record
    TokenProb: PSingle;
    RowFlags: PInt32;
    CandIds: PInt32;
    CandProbs: PSingle;
    CandStride: Int32;
    PhaseMask: Int32;   { 0; G4S_PHASE_FULL_STREAM_ONLY = 1 times the streaming pass alone }
    FullProbs: PSingle;
  end;
  PG4SOutputs = ^TG4SOutputs;

  PG4SCtx = Pointer;

  { TTensorInfo (src/Gemma4.Types.pas:119-129) as g4s_tensor_info. }
  TG4STensorInfo = record
    Name: array[0..255] of AnsiChar;
    SourceDtype: Int32;
    OutputDtype: Int32;
    Offset: UInt64;
    Size: UInt64;
    NDim: Int32;
    Shape: array[0..7] of Int64;
  end;
  PG4STensorInfo = ^TG4STensorInfo;
  PG4SVpk = Pointer;

function g4s_version(): Int32; cdecl; external G4SLib;
procedure g4s_params_defaults(P: PG4SParams); cdecl; external G4SLib;
function g4s_create(Device, MaxRows, MaxVocab: Int32; Flags: UInt32;
  out Ctx: PG4SCtx): Int32; cdecl; external G4SLib;
function g4s_destroy(Ctx: PG4SCtx): Int32; cdecl; external G4SLib;
function g4s_last_error(Ctx: PG4SCtx): PAnsiChar; cdecl; external G4SLib;
function g4s_stream(Ctx: PG4SCtx): Pointer; cdecl; external G4SLib;
function g4s_workspace_bytes(Ctx: PG4SCtx): Int64; cdecl; external G4SLib;

{ Device-pointer form (logits, U and OutTokens in GPU memory; Params on the host). }
function g4s_sample(Ctx: PG4SCtx; Logits: Pointer; DType, Rows, Vocab: Int32;
  RowStride: Int64; Params: PG4SParams; ParamsStride: Int32; Softcap: Single;
  U: PDouble; OutTokens: PInt32; Stream: Pointer): Int32; cdecl; external G4SLib;
function g4s_sample_ex(Ctx: PG4SCtx; Logits: Pointer; DType, Rows, Vocab: Int32;
  RowStride: Int64; Params: PG4SParams; ParamsStride: Int32; Softcap: Single;
  U: PDouble; OutTokens: PInt32; Extra: PG4SOutputs;
  Stream: Pointer): Int32; cdecl; external G4SLib;

{ Host-memory form: the literal drop-in for DoSample on FLogits (synchronous). }
function g4s_sample_host(Ctx: PG4SCtx; HostLogits: Pointer; DType, Rows,
  Vocab: Int32; RowStride: Int64; Params: PG4SParams; ParamsStride: Int32;
  Softcap: Single; HostU: PDouble; HostTokens: PInt32): Int32; cdecl;
  external G4SLib;

{ Top-K sampling without a context or any allocation (static scratch). }
function g4s_sample_topk_noalloc(Logits: Pointer; DType, Rows, Vocab: Int32;
  RowStride: Int64; Params: PG4SParams; Softcap: Single; U: PDouble;
  OutTokens: PInt32; Stream: Pointer): Int32; cdecl; external G4SLib;

{ G4S_ERR_TIMEOUT when a kernel gave up a bounded wait since the last check. }
function g4s_device_status(Ctx: PG4SCtx): Int32; cdecl; external G4SLib;

{ Test hook: Polls > 0 makes the streaming top-K pass's bounded waits give up
  after that many polls (0 = normal limits). }
function g4s_set_wait_limit(Ctx: PG4SCtx; Polls: Int64): Int32; cdecl;
  external G4SLib;

{ LM head (CpuMatVecQ4, src/Gemma4.Tensors.pas:546-590) + DoSample: TQ4Block
  weights repacked once on the device, then one call per step. }
function g4s_q4_repack(Blocks: Pointer; Vocab, Hidden: Int32; Nibbles: Pointer;
  Scales: Pointer; Stream: Pointer): Int32; cdecl; external G4SLib;
function g4s_lmhead_sample(Ctx: PG4SCtx; Hidden: PSingle; Rows, HiddenSize: Int32;
  NormWeight: PSingle; NormEps: Single;
  Nibbles: Pointer; Scales: Pointer; Vocab: Int32; Params: PG4SParams;
  ParamsStride: Int32; Softcap: Single; U: PDouble; OutTokens: PInt32;
  Extra: PG4SOutputs; OutLogits: PSingle; Stream: Pointer): Int32; cdecl;
  external G4SLib;

{ Vocabulary-sharded mode: compute phases (any collective) and the NCCL form. }
function g4s_shard_lists(Ctx: PG4SCtx; Logits: Pointer; DType, Rows, SliceVocab: Int32;
  RowStride: Int64; IdOffset, VocabTotal: Int32; Params: PG4SParams;
  ParamsStride: Int32; Softcap: Single; OutLists: Pointer; OutCounts: PInt32;
  Stream: Pointer): Int32; cdecl; external G4SLib;
function g4s_shard_merge(Ctx: PG4SCtx; Lists: Pointer; Counts: PInt32;
  World, Rows, VocabTotal: Int32; Params: PG4SParams; ParamsStride: Int32;
  Softcap: Single; U: PDouble; OutTokens: PInt32; Extra: PG4SOutputs;
  Stream: Pointer): Int32; cdecl; external G4SLib;
function g4s_shard_resolve(Ctx: PG4SCtx; LogitsSlice: Pointer; DType, Rows,
  SliceVocab: Int32; RowStride: Int64; IdOffset, Rank: Int32; Params: PG4SParams;
  ParamsStride: Int32; Softcap: Single; U: PDouble; OutTokens: PInt32;
  Extra: PG4SOutputs; Stream: Pointer): Int32; cdecl; external G4SLib;
function g4s_shard_unique_id(Uid: PByte): Int32; cdecl; external G4SLib;
function g4s_shard_set_timeout(Ctx: PG4SCtx; Ms: Int64): Int32; cdecl; external G4SLib;
function g4s_shard_wait(Ctx: PG4SCtx; Stream: Pointer; TimeoutMs: Int64): Int32;
  cdecl; external G4SLib;
function g4s_shard_abort(Ctx: PG4SCtx): Int32; cdecl; external G4SLib;
function g4s_shard_init(Ctx: PG4SCtx; World, Rank, VocabTotal: Int32;
  Uid: PByte): Int32; cdecl; external G4SLib;
function g4s_shard_sample(Ctx: PG4SCtx; LogitsSlice: Pointer; DType, Rows: Int32;
  RowStride: Int64; Params: PG4SParams; ParamsStride: Int32; Softcap: Single;
  U: PDouble; OutTokens: PInt32; Extra: PG4SOutputs;
  Stream: Pointer): Int32; cdecl; external G4SLib;

{ The VPK weight archive (TWeightStore): open, look up, read, load the LM head. }
function g4s_vpk_open(Path, ManifestPath, WeightsPath: PAnsiChar;
  out Vpk: PG4SVpk): Int32; cdecl; external G4SLib;
function g4s_vpk_close(Vpk: PG4SVpk): Int32; cdecl; external G4SLib;
function g4s_vpk_tensor_count(Vpk: PG4SVpk): Int32; cdecl; external G4SLib;
function g4s_vpk_tensor_at(Vpk: PG4SVpk; Index: Int32;
  Info: PG4STensorInfo): Int32; cdecl; external G4SLib;
function g4s_vpk_find(Vpk: PG4SVpk; Name: PAnsiChar;
  Info: PG4STensorInfo): Int32; cdecl; external G4SLib;
function g4s_vpk_data(Vpk: PG4SVpk; Info: PG4STensorInfo): Pointer; cdecl;
  external G4SLib;
function g4s_vpk_verify(Vpk: PG4SVpk; EntryPath: PAnsiChar): Int32; cdecl;
  external G4SLib;
function g4s_vpk_load_lmhead(Vpk: PG4SVpk; Device: Int32; Nibbles: Pointer;
  Scales: Pointer; MaxVocab: Int32; out Vocab, Hidden: Int32;
  Stream: Pointer): Int32; cdecl; external G4SLib;

implementation

end.
