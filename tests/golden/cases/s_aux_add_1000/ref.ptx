.version 8.0
.target sm_89
.address_size 64

.visible .entry k_add_aux(
        .param .u64 param_a,
        .param .u64 param_b,
        .param .u64 param_c
)
.reqntid 32, 5, 1
{
        .reg .pred      %p<2>;
        .reg .f32       %f<4>;
        .reg .b32       %r<21>;
        .reg .b64       %rd<7>;

        ld.param.u64    %rd1, [param_a];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_b];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_c];
        cvta.to.global.u64     %rd3, %rd3;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mov.u32         %r5, %tid.y;
        mov.u32         %r6, %tid.z;
        mov.u32         %r7, %ntid.y;
        mov.u32         %r8, %ntid.z;
        mov.u32         %r11, %ctaid.y;
        mov.u32         %r12, %ctaid.z;
        mov.u32         %r9, %nctaid.x;
        mov.u32         %r10, %nctaid.y;
        mad.lo.s32      %r16, %r6, %r7, %r5;
        mad.lo.s32      %r13, %r16, %r2, %r1;
        mad.lo.s32      %r16, %r12, %r10, %r11;
        mad.lo.s32      %r14, %r16, %r9, %r3;
        mul.lo.s32      %r16, %r2, %r7;
        mul.lo.s32      %r15, %r16, %r8;
        mad.lo.s32      %r4, %r14, %r15, %r13;
        mov.u32         %r17, %nctaid.z;
        mul.lo.s32      %r18, %r9, %r10;
        mul.lo.s32      %r18, %r18, %r17;
        rem.s32         %r19, %r13, 128;
        mad.lo.s32      %r20, %r14, 128, %r19;
        setp.ge.s32     %p1, %r20, 1000;
        @%p1 bra        SKIP_1;
        mad.wide.s32    %rd4, %r20, 4, %rd1;
        ld.global.nc.f32   %f1, [%rd4];
        mad.wide.s32    %rd5, %r20, 4, %rd2;
        ld.global.nc.f32   %f2, [%rd5];
        add.f32         %f3, %f1, %f2;
        mad.wide.s32    %rd6, %r20, 4, %rd3;
        st.global.f32   [%rd6], %f3;
SKIP_1:
        ret;
}
