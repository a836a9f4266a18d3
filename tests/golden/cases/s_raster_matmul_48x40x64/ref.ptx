.version 8.0
.target sm_89
.address_size 64

.visible .entry k_matmul_raster(
        .param .u64 param_A,
        .param .u64 param_B,
        .param .u64 param_C
)
.reqntid 128
{
        .reg .pred      %p<2>;
        .reg .f32       %f<4>;
        .reg .b32       %r<18>;
        .reg .b64       %rd<7>;

        ld.param.u64    %rd1, [param_A];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_B];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_C];
        cvta.to.global.u64     %rd3, %rd3;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        shr.u32         %r6, %r4, 8;
        and.b32         %r7, %r4, 3;
        mad.lo.s32      %r8, %r6, 4, %r7;
        and.b32         %r9, %r4, 255;
        shr.u32         %r10, %r9, 2;
        mov.f32         %f1, 0f00000000;
        mov.s32         %r11, 0;
        .pragma "nounroll";
LOOP_1:
        mul.lo.s32      %r12, %r8, 40;
        add.s32         %r13, %r12, %r11;
        mad.wide.s32    %rd4, %r13, 4, %rd1;
        ld.global.nc.f32   %f2, [%rd4];
        shl.b32         %r14, %r11, 6;
        add.s32         %r15, %r14, %r10;
        mad.wide.s32    %rd5, %r15, 4, %rd2;
        ld.global.nc.f32   %f3, [%rd5];
        fma.rn.f32      %f1, %f2, %f3, %f1;
        add.s32         %r11, %r11, 1;
        setp.lt.s32     %p1, %r11, 40;
        @%p1 bra        LOOP_1;
        shl.b32         %r16, %r8, 6;
        add.s32         %r17, %r16, %r10;
        mad.wide.s32    %rd6, %r17, 4, %rd3;
        st.global.f32   [%rd6], %f1;
        ret;
}
