// Substitute for the executable decode_dispatch_12 of model/qwen3_full.mlir
// (iree-compile --iree-hal-substitute-executable-source=decode_dispatch_12=<this
// file>, with --iree-hal-executable-object-search-path naming the directory
// of q3_dispatch.ptx; `make -C qwen3-iree_b200 iree` builds it for sm_100a).
// The export keeps the interface of the substituted executable: 2 push
// constants, bindings b0 (ReadOnly), b1 (ReadOnly|Indirect), b2 (Indirect);
// a fixed grid of 128 workgroups of 256 threads (8 output rows each).
hal.executable public @decode_dispatch_12 {
  hal.executable.variant public @cuda_nvptx_fb target(<"cuda", "cuda-nvptx-fb">) objects([
    #hal.executable.object<{path = "q3_dispatch.ptx"}>
  ]) {
    hal.executable.export public @decode_dispatch_12_matmul_1024x1x2048_f16 ordinal(0) layout(#hal.pipeline.layout<constants = 2, bindings = [#hal.pipeline.binding<storage_buffer, ReadOnly>, #hal.pipeline.binding<storage_buffer, "ReadOnly|Indirect">, #hal.pipeline.binding<storage_buffer, Indirect>], flags = Indirect>) count(%arg0: !hal.device, %arg1: index, %arg2: index) -> (index, index, index) {
      %c128 = arith.constant 128 : index
      %c1 = arith.constant 1 : index
      hal.return %c128, %c1, %c1 : index, index, index
    } attributes {workgroup_size = [256 : index, 1 : index, 1 : index]}
  }
}
