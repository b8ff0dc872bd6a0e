defmodule Transmuter.CUDAQ4 do
  @moduledoc """
  The CUDA (B200) backend of Transmuter's quantized operators, over libtq4 through
  `Transmuter.CUDAQ4.NIF` (c_src/tq4_nif.c). It plugs into `Transmuter.move/2`
  (lib/transmuter.ex:1107-1112) like `Transmuter.EMLX`: `compatible?/1` picks the MatMulNBits
  nodes whose B it holds, `weight/6` turns B, the scales and the zero points into a packed
  handle on the GPU (the "B:packed" value), and `evaluate/1` leaves that handle as it is. At run
  time `Transmuter.Ops.Quantized` calls `matmul/3` when B is a `Transmuter.CUDAQ4.Weight`
  (quantized.ex:39-44), and `gather/3` for GatherBlockQuantized tables (quantized.ex:49-66).

  Device buffers cross the NIF as the device addresses of the EXLA backend's buffers
  (`Nx.to_pointer/2`, Nx 0.9 and later); the kernels are enqueued on the stream given (0: the
  default stream). This module is not compiled in the build container, which has no Elixir: it
  is the binding a maintainer adds, checked there only for its NIF arities.
  """

  alias Transmuter.Ops.Quantized
  alias Transmuter.CUDAQ4.NIF

  @dtypes %{{:f, 32} => 0, {:f, 16} => 1, {:bf, 16} => 2, {:u, 8} => 3, {:s, 8} => 4}
  @zp_none 0
  @zp_packed 1
  @zp_float 2

  defmodule Weight do
    @moduledoc false
    # A packed MatMulNBits weight {N, K} held by libtq4 on `device`, dequantizing in `type`.
    defstruct [:ref, :shape, :type, :device]
  end

  @doc false
  # Every MatMulNBits node libtq4 takes: bits 2, 4 or 8 and power-of-two blocks of 16 or more,
  # K a multiple of the block or not (packable?/2, lib/transmuter.ex:1209-1225, asks for a
  # multiple; the adapter relaxes that for this backend).
  def compatible?(node) do
    {_k, _n, bits, block} = Quantized.nbits_sizes(node)
    bits in [2, 4, 8] and block >= 16 and Bitwise.band(block, block - 1) == 0
  end

  @doc false
  # The handle of a MatMulNBits node: B, the scales and the zero points copied once to the GPU,
  # dequantizing in the scales' type after :compute_type (dequantized_weight/6,
  # lib/transmuter.ex:1230-1240). A deferred initializer (Transmuter.DeferredTensor) is passed as
  # {path, offset, length} and streamed from its file.
  def weight(node, b, scales, zero_points, model, backend) do
    {k, n, bits, block} = Quantized.nbits_sizes(node)
    device = device_index(backend)
    scales = Transmuter.upcast(scales, model[:compute_type])
    t = Map.fetch!(@dtypes, Nx.type(scales))
    {zp_kind, zp_t, zp} = zero_points(zero_points)

    ref =
      NIF.weight_create(k, n, bits, block, t, zp_kind, zp_t, t, 0, source(b), source(scales), zp, device)
      |> ok!()

    %Weight{ref: ref, shape: {n, k}, type: Nx.type(scales), device: device}
  end

  @doc false
  def evaluate(weight), do: weight

  @doc false
  # Sibling MatMulNBits weights merged along N (the packed form of Fusion.matmuls/2,
  # lib/transmuter/fusion.ex:430-540); the caller splits the output with the parts' N.
  def merge(weights = [%Weight{type: type, device: device, shape: {_, k}} | _]) do
    ref = weights |> Enum.map(& &1.ref) |> NIF.weight_merge() |> ok!()
    n = weights |> Enum.map(&elem(&1.shape, 0)) |> Enum.sum()
    %Weight{ref: ref, shape: {n, k}, type: type, device: device}
  end

  @doc false
  # Y = A . W^T (+ bias) for A {..., K} on the weight's device (quantized.ex:39-45). Decode calls
  # (at most 16 rows) with `noalloc: true` allocate no device memory (matmul_noalloc).
  def matmul(a, %Weight{ref: ref, shape: {n, k}}, bias, opts \\ []) do
    shape = Nx.shape(a)
    ^k = elem(shape, tuple_size(shape) - 1)
    m = div(Nx.size(a), k)
    y = Nx.broadcast(Nx.tensor(0, type: Nx.type(a)), put_elem(shape, tuple_size(shape) - 1, n))
    {bias_ptr, bias_t} = if bias, do: {address(bias), Map.fetch!(@dtypes, Nx.type(bias))}, else: {0, 0}
    stream = Keyword.get(opts, :stream, 0)
    call = if Keyword.get(opts, :noalloc, false) and m <= 16, do: &NIF.matmul_noalloc/9, else: &NIF.matmul/9
    :ok = call.(ref, address(a), m, Map.fetch!(@dtypes, Nx.type(a)), bias_ptr, bias_t, address(y),
             Map.fetch!(@dtypes, Nx.type(a)), stream) |> ok!()
    y
  end

  @doc false
  # GatherBlockQuantized (quantized.ex:49-66): rows `indices` of a table held as a weight whose
  # "N" rows are the table's rows, dequantized in its scales' type.
  def gather(%Weight{ref: ref, shape: {_rows, k}, type: type}, indices, opts \\ []) do
    idx = Nx.as_type(indices, :s64)
    out = Nx.broadcast(Nx.tensor(0, type: type), Tuple.append(Nx.shape(idx), k))
    :ok = NIF.gather_rows(ref, address(idx), Nx.size(idx), address(out), Keyword.get(opts, :stream, 0)) |> ok!()
    out
  end

  defp zero_points(nil), do: {@zp_none, 3, nil}

  defp zero_points(zp) do
    type = Nx.type(zp)
    kind = if Nx.Type.float?(type), do: @zp_float, else: @zp_packed
    {kind, Map.fetch!(@dtypes, type), source(zp)}
  end

  # A deferred initializer as {path, offset, length} (the entries Ops.read_external/2 reads,
  # lib/transmuter/ops.ex:680-695; length -1 reads to the end of the file), else its bytes.
  defp source(%Transmuter.DeferredTensor{proto: %{external_data: entries}, dir: dir}) do
    entries = Map.new(entries, &{&1.key, &1.value})
    offset = String.to_integer(entries["offset"] || "0")
    length = if l = entries["length"], do: String.to_integer(l), else: -1
    {String.to_charlist(Path.join(dir, entries["location"])), offset, length}
  end

  defp source(t), do: Nx.to_binary(t)

  defp address(tensor) do
    %{address: address} = Nx.to_pointer(tensor, mode: :local)
    address
  end

  defp device_index({_module, opts}), do: Keyword.get(opts, :device_id, 0)
  defp device_index(_backend), do: 0

  defp ok!(:ok), do: :ok
  defp ok!({:ok, value}), do: value
  defp ok!({:error, message}), do: raise(ArgumentError, List.to_string(message))
end
