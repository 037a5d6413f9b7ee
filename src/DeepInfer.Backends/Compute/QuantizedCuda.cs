using System.Runtime.InteropServices;
using Microsoft.Win32.SafeHandles;
namespace DeepInfer.Backends.Compute;

// CUDA (B200, sm_100a) twin of QuantizedMetal (src/DeepInfer.Backends/Compute/QuantizedMetal.cs).
// The operator half (Allocate, MultiplyBatch, ExpertMlp, QuantMatrix-style Write/Multiply/CopyRow) keeps
// QuantizedMetal's managed checks and binds the same di_quant_* entries in libdeepinfer_cuda.so; the
// native side repeats every check and returns the same error texts. The MoE half binds the batched
// block entries (router -> top-8 -> expert-grouped GEMMs -> shared expert -> combine) that replace
// Qwen36Model.Moe's per-token loop (Qwen36Model.cs:218-262), checkpoint loading of a layer's eight
// matrices (Qwen36Weights.cs:55-100) and the expert-parallel group. Every entry declared in
// include/deepinfer_cuda.h is bound exactly once in CudaQuantNative; tests/test_csharp_twin.py checks
// the names and parameter counts against the header.
public sealed unsafe class QuantizedCuda : IDisposable
{
    internal const int ErrorCapacity = 2048;
    internal readonly CudaHandle Context;
    public long Dispatches { get; private set; }
    public long Submissions { get; private set; }
    public double GpuMilliseconds { get; private set; }

    public QuantizedCuda(bool? residency = null, int residencyRefreshMilliseconds = 1000)
    {
        if (residencyRefreshMilliseconds is < 0 or > 60000) throw new ArgumentOutOfRangeException(nameof(residencyRefreshMilliseconds));
        if (CudaQuantNative.AbiVersion() != 1) throw new InvalidOperationException("deepinfer_cuda ABI version mismatch.");
        var error = new byte[ErrorCapacity];
        fixed (byte* e = error)
        {
            var p = residency is bool on
                ? CudaQuantNative.CreateConfigured(on ? 1 : 0, residencyRefreshMilliseconds, e, error.Length)
                : CudaQuantNative.Create(e, error.Length);
            if (p == 0) throw new InvalidOperationException(Text(error));
            Context = new(p, CudaHandle.Kind.Context);
        }
    }

    public ulong ResidencyBytes => CudaQuantNative.ResidencyBytes(Context);
    public void PrepareResidency() => CudaQuantNative.PrepareResidency(Context);

    public CudaQuantMatrix Allocate(int experts, int rows, int columns, int bits, int group = 64)
    {
        ObjectDisposedException.ThrowIf(Context.IsClosed, this);
        if (experts is < 1 or > 256 || rows is < 1 or > 262144 || columns is < 64 or > 32768 ||
            columns % 64 != 0 || bits is not (5 or 8) || group != 64)
            throw new ArgumentException("Unsupported quantized shape/precision.");
        _ = checked(experts * rows * (columns * bits / 8));
        var error = new byte[ErrorCapacity];
        fixed (byte* e = error)
        {
            var p = CudaQuantNative.MatrixCreate(Context, experts, rows, columns, bits, group, e, error.Length);
            if (p == 0) throw new InvalidOperationException(Text(error));
            return new(this, new(p, CudaHandle.Kind.Matrix), experts, rows, columns, bits);
        }
    }

    // Independent GEMV jobs in one submission (the distinctness rule of QuantizedMetal.MultiplyBatch).
    public void MultiplyBatch(ReadOnlySpan<CudaQuantizedJob> jobs)
    {
        ObjectDisposedException.ThrowIf(Context.IsClosed, this);
        if (jobs.Length is < 1 or > 8) throw new ArgumentException("Expected 1..8 independent GEMV jobs.");
        ReadOnlySpan<int> single = [0];
        for (var i = 0; i < jobs.Length; i++)
        {
            var job = jobs[i];
            if (job.Matrix is null || job.Input is null || job.Output is null) throw new ArgumentException("Incomplete GEMV job.");
            if (!ReferenceEquals(job.Matrix.Owner, this)) throw new ArgumentException("Batch matrices must belong to this device.");
            job.Matrix.Validate(job.Input.Length, job.Output.Length, job.Experts ?? single, job.Batched);
            for (var j = 0; j < i; j++)
            {
                var other = jobs[j];
                if (ReferenceEquals(job.Matrix, other.Matrix) || ReferenceEquals(job.Output, other.Output) ||
                    ReferenceEquals(job.Output, other.Input) || ReferenceEquals(job.Input, other.Output))
                    throw new ArgumentException("GEMV jobs must have distinct matrices/outputs and no cross-job dependencies.");
            }
        }
        var native = new CudaQuantNative.Job[jobs.Length];
        var pins = new List<GCHandle>(jobs.Length * 3);
        var held = new List<CudaHandle>(jobs.Length);
        int[] zero = [0];
        try
        {
            for (var i = 0; i < jobs.Length; i++)
            {
                var job = jobs[i];
                var added = false;
                job.Matrix.Handle.DangerousAddRef(ref added);
                if (added) held.Add(job.Matrix.Handle);
                var experts = job.Experts ?? zero;
                var pin = (object o) => { var h = GCHandle.Alloc(o, GCHandleType.Pinned); pins.Add(h); return h.AddrOfPinnedObject(); };
                native[i] = new()
                {
                    Matrix = job.Matrix.Handle.DangerousGetHandle(),
                    Input = (float*)pin(job.Input), Output = (float*)pin(job.Output), Experts = (int*)pin(experts),
                    Count = experts.Length, Batched = job.Batched ? 1 : 0,
                };
            }
            var error = new byte[ErrorCapacity];
            fixed (CudaQuantNative.Job* j = native) fixed (byte* e = error)
            {
                if (CudaQuantNative.Batch(Context, j, native.Length, out var ms, e, error.Length) != 0)
                    throw new InvalidOperationException(Text(error));
                Count(ms, jobs.Length);
            }
        }
        finally
        {
            foreach (var h in pins) h.Free();
            foreach (var h in held) h.DangerousRelease();
        }
    }

    // gate/up + SwiGLU + down for the selected experts plus the independent shared-expert down projection.
    public void ExpertMlp(CudaQuantMatrix gate, CudaQuantMatrix up, CudaQuantMatrix down, CudaQuantMatrix sharedDown,
        ReadOnlySpan<float> input, ReadOnlySpan<float> sharedInput, ReadOnlySpan<int> experts,
        Span<float> expertOutput, Span<float> sharedOutput)
    {
        ObjectDisposedException.ThrowIf(Context.IsClosed, this);
        CudaQuantMatrix[] all = [gate, up, down, sharedDown];
        for (var i = 0; i < all.Length; i++)
        {
            if (all[i] is null || !ReferenceEquals(all[i].Owner, this)) throw new ArgumentException("Expert matrices must belong to this device.");
            for (var j = 0; j < i; j++) if (ReferenceEquals(all[i], all[j])) throw new ArgumentException("Expert matrices must be distinct.");
        }
        if (gate.Rows != up.Rows || gate.Columns != up.Columns || gate.Experts != up.Experts || gate.Bits != up.Bits ||
            down.Columns != gate.Rows || down.Rows != gate.Columns || down.Experts != gate.Experts ||
            sharedDown.Experts != 1 || sharedDown.Rows != down.Rows || ((ReadOnlySpan<float>)expertOutput).Overlaps(sharedOutput))
            throw new ArgumentException("Incompatible expert shapes/precision or overlapping outputs.");
        gate.Validate(input.Length, gate.Rows * experts.Length, experts, false);
        up.Validate(input.Length, up.Rows * experts.Length, experts, false);
        down.Validate(gate.Rows * experts.Length, expertOutput.Length, experts, true);
        sharedDown.Validate(sharedInput.Length, sharedOutput.Length, [0], false);
        var error = new byte[ErrorCapacity];
        fixed (float* x = input) fixed (float* sx = sharedInput) fixed (int* ids = experts)
        fixed (float* y = expertOutput) fixed (float* sy = sharedOutput) fixed (byte* e = error)
        {
            if (CudaQuantNative.Experts(Context, gate.Handle, up.Handle, down.Handle, sharedDown.Handle,
                    x, sx, ids, experts.Length, y, sy, out var ms, e, error.Length) != 0)
                throw new InvalidOperationException(Text(error));
            Count(ms, 3);
        }
    }

    // One MoE block's eight matrices: router [1,E,D] 8-bit, gate/up [E,I,D], down [E,D,I], shared gate/up
    // [1,I,D], shared down [1,D,I], shared route [1,1,D] 8-bit (Qwen36Weights.cs:93-100).
    public CudaMoeLayer CreateMoeLayer(CudaQuantMatrix router, CudaQuantMatrix gate, CudaQuantMatrix up, CudaQuantMatrix down,
        CudaQuantMatrix sharedGate, CudaQuantMatrix sharedUp, CudaQuantMatrix sharedDown, CudaQuantMatrix sharedRoute)
    {
        ObjectDisposedException.ThrowIf(Context.IsClosed, this);
        foreach (var m in new[] { router, gate, up, down, sharedGate, sharedUp, sharedDown, sharedRoute })
            if (m is null || !ReferenceEquals(m.Owner, this)) throw new ArgumentException("Layer matrices must belong to this device.");
        var error = new byte[ErrorCapacity];
        fixed (byte* e = error)
        {
            var p = CudaQuantNative.LayerCreate(Context, router.Handle, gate.Handle, up.Handle, down.Handle,
                sharedGate.Handle, sharedUp.Handle, sharedDown.Handle, sharedRoute.Handle, e, error.Length);
            if (p == 0) throw new InvalidOperationException(Text(error));
            return new(this, new(p, CudaHandle.Kind.Layer), gate.Experts, gate.Columns, gate.Rows);
        }
    }

    // Validates layer `layer` of an MLX checkpoint directory without touching the GPU.
    public static (int Experts, int Hidden, int Intermediate, int Bits) ProbeCheckpoint(string directory, int layer)
    {
        var geometry = new int[4];
        var error = new byte[ErrorCapacity];
        fixed (int* g = geometry) fixed (byte* e = error)
            if (CudaQuantNative.CheckpointProbe(directory, layer, g, e, error.Length) != 0)
                throw new InvalidOperationException(Text(error));
        return (geometry[0], geometry[1], geometry[2], geometry[3]);
    }

    // Loads layer `layer`'s block (the layer owns its matrices); norm receives post_attention_layernorm.weight.
    public CudaMoeLayer LoadMoeLayer(string directory, int layer, Span<float> norm)
    {
        ObjectDisposedException.ThrowIf(Context.IsClosed, this);
        var (experts, hidden, intermediate, _) = ProbeCheckpoint(directory, layer);
        if (norm.Length != hidden) throw new ArgumentException("RMSNorm weight length must equal the hidden size.");
        var error = new byte[ErrorCapacity];
        fixed (float* n = norm) fixed (byte* e = error)
        {
            var p = CudaQuantNative.LayerLoad(Context, directory, layer, n, e, error.Length);
            if (p == 0) throw new InvalidOperationException(Text(error));
            return new(this, new(p, CudaHandle.Kind.Layer), experts, hidden, intermediate);
        }
    }

    // y = sigmoid(x . w_sr) * shared(x) + sum_j p_j * expert_{ids_j}(x) for `tokens` bf16 rows (host memory).
    // ids/probs receive the routing (8 per token) for routeTrace; with MoeFlags.ForceRoutes ids is an input.
    public void MoeBlock(CudaMoeLayer layer, ReadOnlySpan<ushort> x, int tokens, Span<ushort> y,
        Span<int> ids, Span<float> probs, MoeFlags flags = MoeFlags.None)
    {
        layer.CheckOwner(this);
        if ((flags & MoeFlags.DeviceIO) != 0) throw new ArgumentException("Host spans cannot be device pointers.");
        if (tokens is < 1 or > 65536 || x.Length != tokens * layer.Hidden || y.Length != tokens * layer.Hidden ||
            (!ids.IsEmpty && ids.Length != tokens * 8) || (!probs.IsEmpty && probs.Length != tokens * 8) ||
            ((flags & MoeFlags.ForceRoutes) != 0 && ids.IsEmpty))
            throw new ArgumentException("MoE block input/output shape mismatch.");
        var error = new byte[ErrorCapacity];
        fixed (ushort* xp = x) fixed (ushort* yp = y) fixed (int* ip = ids) fixed (float* pp = probs) fixed (byte* e = error)
        {
            if (CudaQuantNative.Block(Context, layer.Handle, xp, tokens, yp, ip, pp, (int)flags, out var ms, e, error.Length) != 0)
                throw new InvalidOperationException(Text(error));
            Count(ms);
        }
    }

    // Stacked blocks over an f32 residual stream: h = bf16(RMSNorm(x) * norms[l]); x += block_l(h).
    public void MoeStack(ReadOnlySpan<CudaMoeLayer> layers, ReadOnlySpan<float> norms, float eps, Span<float> x, int tokens,
        Span<ushort> hTrace = default, Span<int> idsTrace = default, MoeFlags flags = MoeFlags.None)
    {
        if (layers.Length < 1) throw new ArgumentException("Expected at least one layer.");
        var hidden = layers[0].Hidden;
        foreach (var l in layers) { l.CheckOwner(this); if (l.Hidden != hidden) throw new ArgumentException("Layers must share the hidden size."); }
        if ((flags & (MoeFlags.DeviceIO | MoeFlags.ForceRoutes)) != 0) throw new ArgumentException("Unsupported stack flags.");
        if (tokens < 1 || x.Length != tokens * hidden || norms.Length != layers.Length * hidden ||
            (!hTrace.IsEmpty && hTrace.Length != layers.Length * tokens * hidden) ||
            (!idsTrace.IsEmpty && idsTrace.Length != layers.Length * tokens * 8))
            throw new ArgumentException("MoE stack input/output shape mismatch.");
        var handles = Hold(layers, out var held);
        try
        {
            var error = new byte[ErrorCapacity];
            fixed (nint* lp = handles) fixed (float* np = norms) fixed (float* xp = x) fixed (ushort* hp = hTrace)
            fixed (int* ip = idsTrace) fixed (byte* e = error)
            {
                if (CudaQuantNative.Stack(Context, lp, np, layers.Length, eps, xp, tokens, hp, ip, (int)flags, out var ms, e, error.Length) != 0)
                    throw new InvalidOperationException(Text(error));
                Count(ms, layers.Length);
            }
        }
        finally { foreach (var h in held) h.DangerousRelease(); }
    }

    // The allocation-free block on device memory (x, y, ids, probs are device addresses of this
    // context's GPU; ids/probs may be 0): tokens <= 16, tokens * hidden <= 49152.
    public void MoeBlockStatic(CudaMoeLayer layer, nint x, int tokens, nint y, nint ids, nint probs)
    {
        layer.CheckOwner(this);
        if (tokens is < 1 or > 16 || x == 0 || y == 0) throw new ArgumentException("Invalid allocation-free block call.");
        var error = new byte[ErrorCapacity];
        fixed (byte* e = error)
        {
            if (CudaQuantNative.BlockStatic(Context, layer.Handle, (ushort*)x, tokens, (ushort*)y, (int*)ids, (float*)probs,
                    out var ms, e, error.Length) != 0)
                throw new InvalidOperationException(Text(error));
            Count(ms);
        }
    }

    // Per-stage milliseconds of the last block / profiled stack:
    // [router, top8+count, scan, scatter, gate_up, down, combine, rmsnorm].
    public int LastProfile(Span<double> stageMilliseconds)
    {
        fixed (double* s = stageMilliseconds) return CudaQuantNative.LastProfile(Context, s, stageMilliseconds.Length);
    }

    // The expert-grouped permutation of the last grouped-path block (prefill_moe.mm:8-17 order);
    // returns the route count 8T, or -1 when the last call built none.
    public int LastRoutes(Span<int> permutedRoutes, Span<int> segmentOffsets, Span<int> segmentCounts)
    {
        if (segmentOffsets.Length != segmentCounts.Length) throw new ArgumentException("Segment spans must have equal lengths.");
        var error = new byte[ErrorCapacity];
        fixed (int* r = permutedRoutes) fixed (int* o = segmentOffsets) fixed (int* c = segmentCounts) fixed (byte* e = error)
            return CudaQuantNative.LastRoutes(Context, r, o, c, permutedRoutes.Length, e, error.Length);
    }

    internal static nint[] Hold(ReadOnlySpan<CudaMoeLayer> layers, out List<CudaHandle> held)
    {
        held = new(layers.Length);
        var handles = new nint[layers.Length];
        try
        {
            for (var i = 0; i < layers.Length; i++)
            {
                var added = false;
                layers[i].Handle.DangerousAddRef(ref added);
                if (added) held.Add(layers[i].Handle);
                handles[i] = layers[i].Handle.DangerousGetHandle();
            }
        }
        catch { foreach (var h in held) h.DangerousRelease(); throw; }
        return handles;
    }

    internal void Count(double ms, int dispatches = 1, int submissions = 1) { Dispatches += dispatches; Submissions += submissions; GpuMilliseconds += ms; }
    internal static string Text(byte[] bytes) => System.Text.Encoding.UTF8.GetString(bytes).TrimEnd('\0');
    public void Dispose() => Context.Dispose();
}

[Flags]
public enum MoeFlags
{
    None = 0,
    DeviceIO = 1,       // DI_MOE_DEVICE_IO
    ForceRoutes = 2,    // DI_MOE_FORCE_ROUTES
    PathGemv = 4,       // DI_MOE_PATH_GEMV
    PathGrouped = 8,    // DI_MOE_PATH_GROUPED
    Profile = 16,       // DI_MOE_PROFILE
    RouterExact = 32,   // DI_MOE_ROUTER_EXACT
}

public readonly record struct CudaQuantizedJob(CudaQuantMatrix Matrix, float[] Input, float[] Output, int[]? Experts = null, bool Batched = false);

public sealed unsafe class CudaQuantMatrix : IDisposable
{
    private readonly QuantizedCuda owner;
    private readonly CudaHandle handle;
    internal QuantizedCuda Owner => owner;
    internal CudaHandle Handle => handle;
    public int Experts { get; }
    public int Rows { get; }
    public int Columns { get; }
    public int Bits { get; }

    internal CudaQuantMatrix(QuantizedCuda owner, CudaHandle handle, int experts, int rows, int columns, int bits)
    { this.owner = owner; this.handle = handle; Experts = experts; Rows = rows; Columns = columns; Bits = bits; }

    private int BufferBytes(int index) => checked(Experts * Rows * (index == 0 ? Columns * Bits / 8 : Columns / 64 * 2));

    // Host-writable pinned staging buffer; uploaded before the next compute call or at PrepareResidency.
    private Span<byte> Buffer(int index)
    {
        ObjectDisposedException.ThrowIf(handle.IsClosed || owner.Context.IsClosed, this);
        if (index is < 0 or > 2) throw new ArgumentOutOfRangeException(nameof(index));
        var p = CudaQuantNative.MatrixBuffer(handle, index);
        if (p == 0) throw new InvalidOperationException("Missing quantized buffer.");
        return new((void*)p, BufferBytes(index));
    }

    public void Write(int index, ReadOnlySpan<byte> data)
    {
        var buffer = Buffer(index);
        if (buffer.Length != data.Length) throw new ArgumentException("Quantized buffer length mismatch.");
        data.CopyTo(buffer);
    }

    // Direct host -> device copy without the staging buffer (index 0 codes, 1 scales, 2 biases).
    public void Upload(int index, ReadOnlySpan<byte> data)
    {
        ObjectDisposedException.ThrowIf(handle.IsClosed || owner.Context.IsClosed, this);
        var error = new byte[QuantizedCuda.ErrorCapacity];
        fixed (byte* d = data) fixed (byte* e = error)
            if (CudaQuantNative.MatrixUpload(handle, index, d, (ulong)data.Length, e, error.Length) != 0)
                throw new InvalidOperationException(QuantizedCuda.Text(error));
    }

    // Synthetic N(0, stddev) weights quantised on the device (benchmarks); expert e takes stream expert firstExpert + e.
    public void Generate(ulong seed, ulong stream, float stddev, int firstExpert = 0)
    {
        ObjectDisposedException.ThrowIf(handle.IsClosed || owner.Context.IsClosed, this);
        var error = new byte[QuantizedCuda.ErrorCapacity];
        fixed (byte* e = error)
            if (CudaQuantNative.MatrixGenerate(handle, seed, stream, stddev, firstExpert, e, error.Length) != 0)
                throw new InvalidOperationException(QuantizedCuda.Text(error));
    }

    // Device address of buffer `index` for callers that keep activations on the GPU; writes through it
    // are not seen by the library's router-norm cache.
    public nint DeviceBuffer(int index)
    {
        ObjectDisposedException.ThrowIf(handle.IsClosed || owner.Context.IsClosed, this);
        return CudaQuantNative.MatrixDeviceBuffer(handle, index);
    }

    public void Multiply(ReadOnlySpan<float> input, Span<float> output) => MultiplyExperts(input, output, [0]);

    public void MultiplyExperts(ReadOnlySpan<float> input, Span<float> output, ReadOnlySpan<int> experts, bool batched = false)
    {
        Validate(input.Length, output.Length, experts, batched);
        var error = new byte[QuantizedCuda.ErrorCapacity];
        fixed (float* x = input) fixed (float* y = output) fixed (int* ids = experts) fixed (byte* e = error)
        {
            if (CudaQuantNative.MatVec(owner.Context, handle, x, y, ids, experts.Length, batched ? 1 : 0, out var ms, e, error.Length) != 0)
                throw new InvalidOperationException(QuantizedCuda.Text(error));
            owner.Count(ms);
        }
    }

    // Token-batch projection y[t] = W[expert] x[t] on the tensor cores (bf16 rows in and out).
    public void MultiplyTokens(ReadOnlySpan<ushort> input, int tokens, Span<ushort> output, int expert = 0)
    {
        ObjectDisposedException.ThrowIf(handle.IsClosed || owner.Context.IsClosed, this);
        if (tokens < 1 || input.Length != tokens * Columns || output.Length != tokens * Rows || expert < 0 || expert >= Experts)
            throw new ArgumentException("Quantized GEMM input/output shape mismatch.");
        var error = new byte[QuantizedCuda.ErrorCapacity];
        fixed (ushort* x = input) fixed (ushort* y = output) fixed (byte* e = error)
        {
            if (CudaQuantNative.Gemm(owner.Context, handle, expert, x, tokens, y, 0, out var ms, e, error.Length) != 0)
                throw new InvalidOperationException(QuantizedCuda.Text(error));
            owner.Count(ms);
        }
    }

    internal void Validate(int inputLength, int outputLength, ReadOnlySpan<int> experts, bool batched)
    {
        ObjectDisposedException.ThrowIf(handle.IsClosed || owner.Context.IsClosed, this);
        if (experts.Length is < 1 or > 8 || inputLength != Columns * (batched ? experts.Length : 1) || outputLength != Rows * experts.Length)
            throw new ArgumentException("Quantized GEMV input/output shape mismatch.");
        foreach (var id in experts) if (id < 0 || id >= Experts) throw new ArgumentOutOfRangeException(nameof(experts));
    }

    public void CopyRow(int token, Span<float> output)
    {
        ObjectDisposedException.ThrowIf(handle.IsClosed || owner.Context.IsClosed, this);
        if (output.Length != Columns || token < 0 || token >= Rows || Experts != 1) throw new ArgumentException("Invalid embedding row.");
        fixed (float* y = output)
            if (CudaQuantNative.Embedding(handle, token, y) != 0) throw new InvalidOperationException("Embedding lookup failed.");
    }

    public void Dispose() => handle.Dispose();
}

// A bound MoE block. The native layer holds a reference on each of its matrices, so the matrices may be
// disposed before the layer.
public sealed unsafe class CudaMoeLayer : IDisposable
{
    private readonly object owner;
    internal readonly CudaHandle Handle;
    public int Experts { get; }
    public int Hidden { get; }
    public int Intermediate { get; }

    internal CudaMoeLayer(object owner, CudaHandle handle, int experts, int hidden, int intermediate)
    { this.owner = owner; Handle = handle; Experts = experts; Hidden = hidden; Intermediate = intermediate; }

    internal void CheckOwner(object expected)
    {
        ObjectDisposedException.ThrowIf(Handle.IsClosed, this);
        if (!ReferenceEquals(owner, expected)) throw new ArgumentException("Layer belongs to another context.");
    }

    // Optional per-expert logit bias (f32[E]); an empty span clears it.
    public void SetRouterBias(ReadOnlySpan<float> bias)
    {
        ObjectDisposedException.ThrowIf(Handle.IsClosed, this);
        if (!bias.IsEmpty && bias.Length != Experts) throw new ArgumentException("Router bias length must equal the expert count.");
        var error = new byte[QuantizedCuda.ErrorCapacity];
        fixed (float* b = bias) fixed (byte* e = error)
            if (CudaQuantNative.LayerSetRouterBias(Handle, bias.IsEmpty ? null : b, e, error.Length) != 0)
                throw new InvalidOperationException(QuantizedCuda.Text(error));
    }

    public void Dispose() => Handle.Dispose();
}

// Expert parallelism across the GPUs of one node, one process per GPU. Rank 0 calls UniqueId and sends
// the bytes to every other rank out of band; every rank then constructs its group (collective).
public sealed unsafe class CudaExpertParallel : IDisposable
{
    private readonly QuantizedCuda device;
    internal readonly CudaHandle Handle;
    public int Rank { get; }
    public int World { get; }

    public static byte[] UniqueId()
    {
        var id = new byte[128];
        var error = new byte[QuantizedCuda.ErrorCapacity];
        fixed (byte* i = id) fixed (byte* e = error)
            if (CudaQuantNative.EpUniqueId(i, e, error.Length) != 0) throw new InvalidOperationException(QuantizedCuda.Text(error));
        return id;
    }

    public CudaExpertParallel(QuantizedCuda device, ReadOnlySpan<byte> id, int rank, int world)
    {
        if (id.Length != 128 || world is < 1 or > 8 || rank < 0 || rank >= world) throw new ArgumentException("Invalid expert-parallel group.");
        var error = new byte[QuantizedCuda.ErrorCapacity];
        fixed (byte* i = id) fixed (byte* e = error)
        {
            var p = CudaQuantNative.EpCreate(device.Context, i, rank, world, e, error.Length);
            if (p == 0) throw new InvalidOperationException(QuantizedCuda.Text(error));
            Handle = new(p, CudaHandle.Kind.ExpertParallel);
        }
        this.device = device; Rank = rank; World = world;
    }

    // gate/up/down hold this rank's E/World experts; router and shared matrices are full.
    public CudaMoeLayer CreateLayer(CudaQuantMatrix router, CudaQuantMatrix gate, CudaQuantMatrix up, CudaQuantMatrix down,
        CudaQuantMatrix sharedGate, CudaQuantMatrix sharedUp, CudaQuantMatrix sharedDown, CudaQuantMatrix sharedRoute)
    {
        ObjectDisposedException.ThrowIf(Handle.IsClosed, this);
        var error = new byte[QuantizedCuda.ErrorCapacity];
        fixed (byte* e = error)
        {
            var p = CudaQuantNative.EpLayerCreate(Handle, router.Handle, gate.Handle, up.Handle, down.Handle,
                sharedGate.Handle, sharedUp.Handle, sharedDown.Handle, sharedRoute.Handle, e, error.Length);
            if (p == 0) throw new InvalidOperationException(QuantizedCuda.Text(error));
            return new(this, new(p, CudaHandle.Kind.Layer), router.Rows, gate.Columns, gate.Rows);
        }
    }

    // Collective: every rank calls it with the same layers; token counts may differ between ranks.
    public void Stack(ReadOnlySpan<CudaMoeLayer> layers, ReadOnlySpan<float> norms, float eps, Span<float> x, int tokens,
        Span<ushort> hTrace = default, Span<int> idsTrace = default)
    {
        if (layers.Length < 1) throw new ArgumentException("Expected at least one layer.");
        var hidden = layers[0].Hidden;
        foreach (var l in layers) l.CheckOwner(this);
        if (tokens < 0 || x.Length != tokens * hidden || norms.Length != layers.Length * hidden ||
            (!hTrace.IsEmpty && hTrace.Length != layers.Length * tokens * hidden) ||
            (!idsTrace.IsEmpty && idsTrace.Length != layers.Length * tokens * 8))
            throw new ArgumentException("Expert-parallel stack input/output shape mismatch.");
        var handles = QuantizedCuda.Hold(layers, out var held);
        try
        {
            var error = new byte[QuantizedCuda.ErrorCapacity];
            fixed (nint* lp = handles) fixed (float* np = norms) fixed (float* xp = x) fixed (ushort* hp = hTrace)
            fixed (int* ip = idsTrace) fixed (byte* e = error)
            {
                if (CudaQuantNative.EpStack(Handle, lp, np, layers.Length, eps, xp, tokens, hp, ip, 0, out var ms, e, error.Length) != 0)
                    throw new InvalidOperationException(QuantizedCuda.Text(error));
                device.Count(ms, layers.Length);
            }
        }
        finally { foreach (var h in held) h.DangerousRelease(); }
    }

    public void Dispose() => Handle.Dispose();
}

internal sealed class CudaHandle : SafeHandleZeroOrMinusOneIsInvalid
{
    internal enum Kind { Context, Matrix, Layer, ExpertParallel }
    private readonly Kind kind;
    public CudaHandle() : base(true) { }
    internal CudaHandle(nint p, Kind kind) : base(true) { SetHandle(p); this.kind = kind; }
    protected override bool ReleaseHandle()
    {
        switch (kind)
        {
            case Kind.Context: CudaQuantNative.Destroy(handle); break;
            case Kind.Matrix: CudaQuantNative.MatrixDestroy(handle); break;
            case Kind.Layer: CudaQuantNative.LayerDestroy(handle); break;
            default: CudaQuantNative.EpDestroy(handle); break;
        }
        return true;
    }
}

// One LibraryImport per entry of include/deepinfer_cuda.h.
internal static unsafe partial class CudaQuantNative
{
    private const string Lib = "deepinfer_cuda";

    [StructLayout(LayoutKind.Sequential)]
    internal struct Job
    {
        public nint Matrix;
        public float* Input;
        public float* Output;
        public int* Experts;
        public int Count, Batched;
    }

    // Part 1: the QuantNative operator table.
    [LibraryImport(Lib, EntryPoint = "di_abi_version")] internal static partial int AbiVersion();
    [LibraryImport(Lib, EntryPoint = "di_quant_create")] internal static partial nint Create(byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_quant_create_configured")] internal static partial nint CreateConfigured(int resident, int refreshMilliseconds, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_quant_destroy")] internal static partial void Destroy(nint context);
    [LibraryImport(Lib, EntryPoint = "di_quant_residency_bytes")] internal static partial ulong ResidencyBytes(CudaHandle context);
    [LibraryImport(Lib, EntryPoint = "di_quant_residency_prepare")] internal static partial void PrepareResidency(CudaHandle context);
    [LibraryImport(Lib, EntryPoint = "di_quant_matrix_create")] internal static partial nint MatrixCreate(CudaHandle context, int experts, int rows, int columns, int bits, int group, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_quant_matrix_buffer")] internal static partial nint MatrixBuffer(CudaHandle matrix, int index);
    [LibraryImport(Lib, EntryPoint = "di_quant_matrix_destroy")] internal static partial void MatrixDestroy(nint matrix);
    [LibraryImport(Lib, EntryPoint = "di_quant_batch")] internal static partial int Batch(CudaHandle context, Job* jobs, int count, out double ms, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_quant_matvec")] internal static partial int MatVec(CudaHandle context, CudaHandle matrix, float* x, float* y, int* experts, int count, int batched, out double ms, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_quant_experts")] internal static partial int Experts(CudaHandle context, CudaHandle gate, CudaHandle up, CudaHandle down, CudaHandle sharedDown,
        float* input, float* sharedInput, int* experts, int count, float* output, float* sharedOutput, out double ms, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_quant_embedding")] internal static partial int Embedding(CudaHandle matrix, int token, float* y);
    [LibraryImport(Lib, EntryPoint = "di_quant_gemm")] internal static partial int Gemm(CudaHandle context, CudaHandle matrix, int expert, ushort* x, int tokens, ushort* y, int flags, out double ms, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_quant_matrix_device_buffer")] internal static partial nint MatrixDeviceBuffer(CudaHandle matrix, int index);
    [LibraryImport(Lib, EntryPoint = "di_quant_matrix_upload")] internal static partial int MatrixUpload(CudaHandle matrix, int index, void* source, ulong bytes, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_quant_matrix_generate")] internal static partial int MatrixGenerate(CudaHandle matrix, ulong seed, ulong stream, float stddev, int firstExpert, byte* error, int capacity);

    // Part 2: the MoE block.
    [LibraryImport(Lib, EntryPoint = "di_moe_layer_create")] internal static partial nint LayerCreate(CudaHandle context, CudaHandle router, CudaHandle gate, CudaHandle up, CudaHandle down,
        CudaHandle sharedGate, CudaHandle sharedUp, CudaHandle sharedDown, CudaHandle sharedRoute, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_layer_destroy")] internal static partial void LayerDestroy(nint layer);
    [LibraryImport(Lib, EntryPoint = "di_moe_layer_set_router_bias")] internal static partial int LayerSetRouterBias(CudaHandle layer, float* bias, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_checkpoint_probe", StringMarshalling = StringMarshalling.Utf8)] internal static partial int CheckpointProbe(string directory, int layer, int* geometry, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_layer_load", StringMarshalling = StringMarshalling.Utf8)] internal static partial nint LayerLoad(CudaHandle context, string directory, int layer, float* norm, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_block")] internal static partial int Block(CudaHandle context, CudaHandle layer, ushort* x, int tokens, ushort* y, int* ids, float* probs, int flags, out double ms, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_stack")] internal static partial int Stack(CudaHandle context, nint* layers, float* norms, int layerCount, float eps, float* x, int tokens,
        ushort* hTrace, int* idsTrace, int flags, out double ms, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_last_profile")] internal static partial int LastProfile(CudaHandle context, double* stageMs, int count);
    [LibraryImport(Lib, EntryPoint = "di_moe_last_routes")] internal static partial int LastRoutes(CudaHandle context, int* permutedRoutes, int* segmentOffsets, int* segmentCounts, int maxRoutes, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_block_static")] internal static partial int BlockStatic(CudaHandle context, CudaHandle layer, ushort* x, int tokens, ushort* y, int* ids, float* probs, out double ms, byte* error, int capacity);

    // Part 3: expert parallelism.
    [LibraryImport(Lib, EntryPoint = "di_moe_ep_unique_id")] internal static partial int EpUniqueId(byte* id, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_ep_create")] internal static partial nint EpCreate(CudaHandle context, byte* id, int rank, int world, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_ep_destroy")] internal static partial void EpDestroy(nint ep);
    [LibraryImport(Lib, EntryPoint = "di_moe_ep_layer_create")] internal static partial nint EpLayerCreate(CudaHandle ep, CudaHandle router, CudaHandle gate, CudaHandle up, CudaHandle down,
        CudaHandle sharedGate, CudaHandle sharedUp, CudaHandle sharedDown, CudaHandle sharedRoute, byte* error, int capacity);
    [LibraryImport(Lib, EntryPoint = "di_moe_ep_stack")] internal static partial int EpStack(CudaHandle ep, nint* layers, float* norms, int layerCount, float eps, float* x, int tokens,
        ushort* hTrace, int* idsTrace, int flags, out double ms, byte* error, int capacity);
}
