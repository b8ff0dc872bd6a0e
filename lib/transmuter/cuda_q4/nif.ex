defmodule Transmuter.CUDAQ4.NIF do
  @moduledoc false
  # The NIF of c_src/tq4_nif.c (built by c_src/Makefile into priv/tq4_nif.so). Each function is
  # replaced when the library loads; the arities match the C table.
  @on_load :load_nif

  def load_nif do
    path = :filename.join(:code.priv_dir(:transmuter), ~c"tq4_nif")
    :erlang.load_nif(path, 0)
  end

  def weight_create(_k, _n, _bits, _block, _scale_t, _zp_kind, _zp_t, _t, _signed, _b, _scales, _zp, _device), do: :erlang.nif_error(:not_loaded)
  def weight_merge(_refs), do: :erlang.nif_error(:not_loaded)
  def matmul(_ref, _a, _m, _a_t, _bias, _bias_t, _y, _y_t, _stream), do: :erlang.nif_error(:not_loaded)
  def matmul_noalloc(_ref, _a, _m, _a_t, _bias, _bias_t, _y, _y_t, _stream), do: :erlang.nif_error(:not_loaded)
  def dequantize(_ref, _out, _stream), do: :erlang.nif_error(:not_loaded)
  def gather_rows(_ref, _indices, _count, _out, _stream), do: :erlang.nif_error(:not_loaded)
  def device_status(_device), do: :erlang.nif_error(:not_loaded)
end
