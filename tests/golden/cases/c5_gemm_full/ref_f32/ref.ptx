.version 8.0
.target sm_89
.address_size 64

.visible .entry k_matmul_bias_relu(
        .param .u64 param_A,
        .param .u64 param_B,
        .param .u64 param_bias,
        .param .u64 param_C
)
.reqntid 128
{
        .reg .pred      %p<2>;
        .reg .f32       %f<7>;
        .reg .b32       %r<15>;
        .reg .b64       %rd<9>;

        ld.param.u64    %rd1, [param_A];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_B];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_bias];
        cvta.to.global.u64     %rd3, %rd3;
        ld.param.u64    %rd4, [param_C];
        cvta.to.global.u64     %rd4, %rd4;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        shr.u32         %r6, %r4, 14;
        and.b32         %r7, %r4, 16383;
        mov.f32         %f1, 0f00000000;
        mov.s32         %r8, 0;
        .pragma "nounroll";
LOOP_1:
        shl.b32         %r9, %r6, 13;
        add.s32         %r10, %r9, %r8;
        mad.wide.s32    %rd5, %r10, 4, %rd1;
        ld.global.nc.f32   %f2, [%rd5];
        shl.b32         %r11, %r8, 14;
        add.s32         %r12, %r11, %r7;
        mad.wide.s32    %rd6, %r12, 4, %rd2;
        ld.global.nc.f32   %f3, [%rd6];
        fma.rn.f32      %f1, %f2, %f3, %f1;
        add.s32         %r8, %r8, 1;
        setp.lt.s32     %p1, %r8, 8192;
        @%p1 bra        LOOP_1;
        mad.wide.s32    %rd7, %r7, 4, %rd3;
        ld.global.nc.f32   %f4, [%rd7];
        add.f32         %f5, %f1, %f4;
        max.f32         %f6, %f5, 0f00000000;
        shl.b32         %r13, %r6, 14;
        add.s32         %r14, %r13, %r7;
        mad.wide.s32    %rd8, %r14, 4, %rd4;
        st.global.f32   [%rd8], %f6;
        ret;
}
