// C# side of the B200 library: the compute backend SharpInfer.Core injects
// (IComputeBackend, src/SharpInfer.Core/Tensors/TensorOps.cs:241-250), its
// quantised extension, and a device-resident model for the decode loop of
// InferenceEngine (src/SharpInfer.Core/Engine/InferenceEngine.cs:71-131).
// All calls go through P/Invoke to libsharpinfer_b200 (include/sharpinfer_b200.h).
//
// Unlike CudaBackend (src/SharpInfer.Gpu/CudaBackend.cs:44-47) there is no
// silent CPU fallback: a missing library or GPU raises, and every non-zero
// si_status becomes a B200Exception carrying si_last_error().
//
// Build: add this file to SharpInfer.Gpu (net8.0, AllowUnsafeBlocks) and put
// libsharpinfer_b200.so next to the application (or on LD_LIBRARY_PATH).
using System;
using System.Runtime.InteropServices;
using SharpInfer.Core.Tensors;

namespace SharpInfer.Gpu;

/// <summary>A failed call into libsharpinfer_b200.</summary>
public sealed class B200Exception : Exception
{
    public int Status { get; }
    public B200Exception(int status, string message) : base($"si_status {status}: {message}") => Status = status;
}

/// <summary>si_model_config (field names of the reference's ModelConfig, Transformer.cs:43-56).</summary>
[StructLayout(LayoutKind.Sequential)]
public struct B200ModelConfig
{
    public int NumLayers, HiddenSize, IntermediateSize, NumAttentionHeads, NumKvHeads, HeadDim, VocabSize;
    public int MaxSequenceLength, MaxBatch;
    public float RmsNormEps, RopeTheta;
    public int WeightType, OutputType, EmbeddingType;  // QuantType values
}

internal static unsafe class B200Native
{
    private const string Lib = "sharpinfer_b200";

    [DllImport(Lib)] public static extern IntPtr si_last_error();
    [DllImport(Lib)] public static extern int si_init(int device, out IntPtr ctx);
    [DllImport(Lib)] public static extern int si_shutdown(IntPtr ctx);
    [DllImport(Lib)] public static extern int si_device_name(IntPtr ctx, byte* buf, int len);
    [DllImport(Lib)] public static extern int si_weight_upload(IntPtr ctx, int qtype, byte* blocks, long rows, long cols, out IntPtr w);
    [DllImport(Lib)] public static extern int si_weight_free(IntPtr w);
    [DllImport(Lib)] public static extern int si_qmatvec_host(IntPtr ctx, IntPtr w, float* x, float* y, int batch);
    [DllImport(Lib)] public static extern int si_qgemm(IntPtr ctx, IntPtr w, ushort* xBf16Dev, float* yDev, int m);
    [DllImport(Lib)] public static extern int si_synchronize(IntPtr ctx);

    [DllImport(Lib)] public static extern int si_model_create(IntPtr ctx, ref B200ModelConfig cfg, out IntPtr model);
    [DllImport(Lib)] public static extern int si_model_free(IntPtr model);
    [DllImport(Lib)] public static extern int si_model_prefill(IntPtr model, int seq, int* tokens, int n, int pos0, int* next, float* logits);
    [DllImport(Lib)] public static extern int si_decode_step(IntPtr model, int* tokens, int batch, int pos, int* next, float* logits);
    [DllImport(Lib)] public static extern int si_decode_generate(IntPtr model, int* tokens, int batch, int pos0, int nsteps, int* outTokens);
    [DllImport(Lib)] public static extern int si_model_kv_export(IntPtr model, int seq, int length, byte* outBytes, nuint outLen);
    [DllImport(Lib)] public static extern int si_model_kv_import(IntPtr model, int seq, int length, byte* inBytes, nuint inLen);

    [DllImport(Lib)] public static extern int si_gguf_open([MarshalAs(UnmanagedType.LPUTF8Str)] string path, out IntPtr g);
    [DllImport(Lib)] public static extern int si_gguf_close(IntPtr g);
    [DllImport(Lib)] public static extern int si_gguf_model_config(IntPtr g, int maxSeq, int maxBatch, out B200ModelConfig cfg);
    [DllImport(Lib)] public static extern int si_model_load_gguf(IntPtr model, IntPtr g);

    // The f32 interface CudaBackend binds (CudaBackend.cs:141-163), same names and signatures.
    [DllImport(Lib)] public static extern void cuda_mat_vec_mul(IntPtr h, float* mat, float* vec, float* res, int rows, int cols);
    [DllImport(Lib)] public static extern void cuda_mat_mul(IntPtr h, float* a, float* b, float* c, int m, int k, int n);
    [DllImport(Lib)] public static extern void cuda_softmax(IntPtr h, float* x, int len);
    [DllImport(Lib)] public static extern void cuda_rms_norm(IntPtr h, float* output, float* x, float* weight, int size, float eps);
    [DllImport(Lib)] public static extern void cuda_silu(IntPtr h, float* x, int len);
    [DllImport(Lib)] public static extern void cuda_add_inplace(IntPtr h, float* a, float* b, int len);

    public static void Check(int status)
    {
        if (status != 0) throw new B200Exception(status, Marshal.PtrToStringUTF8(si_last_error()) ?? "");
    }

    /// <summary>The f32 entry points report failures only through si_last_error.</summary>
    public static void CheckLastError()
    {
        var msg = Marshal.PtrToStringUTF8(si_last_error());
        if (!string.IsNullOrEmpty(msg)) throw new B200Exception(2, msg);
    }
}

/// <summary>A GGUF-quantised weight resident on the GPU (si_weight*).</summary>
public sealed class QuantizedWeight : IDisposable
{
    internal IntPtr Handle;
    public QuantType Type { get; }
    public int Rows { get; }
    public int Cols { get; }
    internal QuantizedWeight(IntPtr h, QuantType type, int rows, int cols) { Handle = h; Type = type; Rows = rows; Cols = cols; }
    public void Dispose()
    {
        if (Handle != IntPtr.Zero) { B200Native.si_weight_free(Handle); Handle = IntPtr.Zero; }
    }
}

/// <summary>
/// The quantised extension of IComputeBackend: weights stay on the device as
/// their GGUF blocks and are dequantised inside the kernels, which the f32
/// spans of IComputeBackend cannot express (they carry dequantised host data
/// across PCIe on every call).
/// </summary>
public interface IQuantizedBackend : IComputeBackend
{
    /// <summary>Raw GGUF blocks of a [rows][cols] tensor (DequantizeTensor's input, Quantization.cs:415-469).</summary>
    QuantizedWeight Upload(QuantType type, ReadOnlySpan<byte> blocks, int rows, int cols);
    /// <summary>y[b][r] = sum_c W[r][c] x[b][c] for b &lt; batch (1..16); MatVecMul without the f32 matrix.</summary>
    void QuantizedMatVec(QuantizedWeight w, ReadOnlySpan<float> x, Span<float> y, int batch);
}

/// <summary>
/// IComputeBackend on a B200: the f32 operations run on the device through
/// the library's f32 interface, the quantised ones through si_*.
/// </summary>
public sealed class B200Backend : IQuantizedBackend, IDisposable
{
    private IntPtr _ctx;
    public int Device { get; }
    public string DeviceName { get; }
    public string Name => $"B200 (Device {Device}: {DeviceName})";
    internal IntPtr Context => _ctx;

    public unsafe B200Backend(int deviceId = 0)
    {
        Device = deviceId;
        B200Native.Check(B200Native.si_init(deviceId, out _ctx));
        var buf = stackalloc byte[256];
        B200Native.Check(B200Native.si_device_name(_ctx, buf, 256));
        DeviceName = Marshal.PtrToStringUTF8((IntPtr)buf) ?? "";
    }

    public unsafe void MatVecMul(ReadOnlySpan<float> mat, ReadOnlySpan<float> vec, Span<float> result, int rows, int cols)
    {
        fixed (float* m = mat, v = vec, r = result) B200Native.cuda_mat_vec_mul(_ctx, m, v, r, rows, cols);
        B200Native.CheckLastError();
    }

    public unsafe void MatMul(ReadOnlySpan<float> a, ReadOnlySpan<float> b, Span<float> c, int M, int K, int N)
    {
        fixed (float* pa = a, pb = b, pc = c) B200Native.cuda_mat_mul(_ctx, pa, pb, pc, M, K, N);
        B200Native.CheckLastError();
    }

    public unsafe void Softmax(Span<float> x)
    {
        fixed (float* p = x) B200Native.cuda_softmax(_ctx, p, x.Length);
        B200Native.CheckLastError();
    }

    public unsafe void RmsNorm(Span<float> output, ReadOnlySpan<float> x, ReadOnlySpan<float> weight, float eps)
    {
        fixed (float* o = output, px = x, w = weight) B200Native.cuda_rms_norm(_ctx, o, px, w, x.Length, eps);
        B200Native.CheckLastError();
    }

    public unsafe void SiLU(Span<float> x)
    {
        fixed (float* p = x) B200Native.cuda_silu(_ctx, p, x.Length);
        B200Native.CheckLastError();
    }

    public unsafe void AddInPlace(Span<float> a, ReadOnlySpan<float> b)
    {
        fixed (float* pa = a, pb = b) B200Native.cuda_add_inplace(_ctx, pa, pb, a.Length);
        B200Native.CheckLastError();
    }

    public unsafe QuantizedWeight Upload(QuantType type, ReadOnlySpan<byte> blocks, int rows, int cols)
    {
        IntPtr w;
        fixed (byte* p = blocks) B200Native.Check(B200Native.si_weight_upload(_ctx, (int)type, p, rows, cols, out w));
        return new QuantizedWeight(w, type, rows, cols);
    }

    public unsafe void QuantizedMatVec(QuantizedWeight w, ReadOnlySpan<float> x, Span<float> y, int batch)
    {
        if (x.Length < batch * w.Cols || y.Length < batch * w.Rows) throw new ArgumentException("span too short");
        fixed (float* px = x, py = y) B200Native.Check(B200Native.si_qmatvec_host(_ctx, w.Handle, px, py, batch));
    }

    public void Dispose()
    {
        if (_ctx != IntPtr.Zero) { B200Native.si_shutdown(_ctx); _ctx = IntPtr.Zero; }
    }
}

/// <summary>
/// A whole model resident on one B200 (si_model*): Transformer.Forward
/// (Transformer.cs:67-162) as one captured CUDA graph per step, the prompt as
/// one batched prefill, the KV cache in f16 on the device.
/// </summary>
public sealed class B200Model : IDisposable
{
    private IntPtr _model;
    public B200ModelConfig Config { get; }

    public B200Model(B200Backend backend, B200ModelConfig config)
    {
        Config = config;
        B200Native.Check(B200Native.si_model_create(backend.Context, ref config, out _model));
    }

    /// <summary>The model of a GGUF file (the loader InferenceEngine.Load expects, InferenceEngine.cs:48-49).</summary>
    public static B200Model LoadGguf(B200Backend backend, string path, int maxSequenceLength = 0)
    {
        B200Native.Check(B200Native.si_gguf_open(path, out var g));
        try
        {
            B200Native.Check(B200Native.si_gguf_model_config(g, maxSequenceLength, 1, out var cfg));
            var model = new B200Model(backend, cfg);
            B200Native.Check(B200Native.si_model_load_gguf(model._model, g));
            return model;
        }
        finally
        {
            B200Native.si_gguf_close(g);
        }
    }

    /// <summary>The prompt at positions startPos.. in one pass (replaces the loop of InferenceEngine.cs:82-85); returns the greedy next token.</summary>
    public unsafe int Prefill(ReadOnlySpan<int> tokens, int startPos, Span<float> logits = default)
    {
        int next;
        fixed (int* t = tokens) fixed (float* l = logits)
            B200Native.Check(B200Native.si_model_prefill(_model, 0, t, tokens.Length, startPos, &next,
                logits.IsEmpty ? null : l));
        return next;
    }

    /// <summary>One Transformer.Forward (Transformer.cs:67-162) with greedy sampling (SamplingPipeline.cs:64-65).</summary>
    public unsafe int Step(int token, int position, Span<float> logits = default)
    {
        int next;
        fixed (float* l = logits)
            B200Native.Check(B200Native.si_decode_step(_model, &token, 1, position, &next, logits.IsEmpty ? null : l));
        return next;
    }

    /// <summary>Greedy tokens decoded on the device, each feeding the next (InferenceEngine.cs:96-131 at Temperature 0).</summary>
    public unsafe int[] Generate(int token, int startPos, int steps)
    {
        var output = new int[steps];
        fixed (int* o = output) B200Native.Check(B200Native.si_decode_generate(_model, &token, 1, startPos, steps, o));
        return output;
    }

    /// <summary>KVCache.WriteRawData's byte format (KVCache.cs:84-98) for PromptCache.</summary>
    public unsafe byte[] ExportKv(int length)
    {
        var bytes = new byte[(long)Config.NumLayers * 2 * length * Config.NumKvHeads * Config.HeadDim * 4];
        fixed (byte* p = bytes) B200Native.Check(B200Native.si_model_kv_export(_model, 0, length, p, (nuint)bytes.Length));
        return bytes;
    }

    /// <summary>KVCache.ReadRawData (KVCache.cs:101-114): values rounded to the f16 cache.</summary>
    public unsafe void ImportKv(ReadOnlySpan<byte> bytes, int length)
    {
        fixed (byte* p = bytes) B200Native.Check(B200Native.si_model_kv_import(_model, 0, length, p, (nuint)bytes.Length));
    }

    public void Dispose()
    {
        if (_model != IntPtr.Zero) { B200Native.si_model_free(_model); _model = IntPtr.Zero; }
    }
}

/// <summary>
/// The greedy path of InferenceEngine.GenerateAsync (InferenceEngine.cs:71-131)
/// on a B200Model: prefill the prompt, then one device step per token until a
/// stop token or the limit.  Tokenisation and text stay with the caller's
/// BpeTokenizer.
/// </summary>
public sealed class B200Generator
{
    private readonly B200Model _model;
    private int _position;

    public B200Generator(B200Model model) => _model = model;

    public System.Collections.Generic.List<int> Generate(ReadOnlySpan<int> promptTokens, int maxTokens, int eosId)
    {
        var produced = new System.Collections.Generic.List<int>();
        int next = _model.Prefill(promptTokens, _position);
        _position += promptTokens.Length;
        for (int step = 0; step < maxTokens && next != eosId; step++)
        {
            produced.Add(next);
            next = _model.Step(next, _position++);
        }
        return produced;
    }
}
