/* embedded_image.S -- links the sm_100a kernel CUBIN (built from
 * kernels/kernels.cu) into libhexir_b200.so as read-only bytes.  The build
 * passes its path as HEXIR_CUBIN. */
  .section .rodata.hexir_cubin, "a"
  .balign 64
  .global hexir_embedded_cubin_begin
  .hidden hexir_embedded_cubin_begin
hexir_embedded_cubin_begin:
  .incbin HEXIR_CUBIN
  .global hexir_embedded_cubin_end
  .hidden hexir_embedded_cubin_end
hexir_embedded_cubin_end:
  .byte 0
  .section .note.GNU-stack, "", @progbits
