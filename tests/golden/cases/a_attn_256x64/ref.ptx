.version 8.0
.target sm_89
.address_size 64

.visible .entry k_attn_naive(
        .param .u64 param_q,
        .param .u64 param_kt,
        .param .u64 param_v,
        .param .u64 param_attn
)
.reqntid 128
{
        .reg .pred      %p<7>;
        .reg .f32       %f<25>;
        .reg .b32       %r<30>;
        .reg .b64       %rd<13>;

        ld.param.u64    %rd1, [param_q];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_kt];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_v];
        cvta.to.global.u64     %rd3, %rd3;
        ld.param.u64    %rd4, [param_attn];
        cvta.to.global.u64     %rd4, %rd4;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        shr.u32         %r6, %r4, 6;
        and.b32         %r7, %r4, 63;
        mov.f32         %f1, 0fF149F2CA;
        mov.s32         %r8, 0;
        .pragma "nounroll";
LOOP_1:
        mov.f32         %f2, 0f00000000;
        mov.s32         %r9, 0;
        .pragma "nounroll";
LOOP_2:
        shl.b32         %r10, %r6, 6;
        add.s32         %r11, %r10, %r9;
        mad.wide.s32    %rd5, %r11, 4, %rd1;
        ld.global.nc.f32   %f3, [%rd5];
        shl.b32         %r12, %r9, 8;
        add.s32         %r13, %r12, %r8;
        mad.wide.s32    %rd6, %r13, 4, %rd2;
        ld.global.nc.f32   %f4, [%rd6];
        fma.rn.f32      %f2, %f3, %f4, %f2;
        add.s32         %r9, %r9, 1;
        setp.lt.s32     %p1, %r9, 64;
        @%p1 bra        LOOP_2;
        mov.f32         %f5, 0f3E000000;
        mul.f32         %f2, %f2, %f5;
        max.f32         %f1, %f1, %f2;
        add.s32         %r8, %r8, 1;
        setp.lt.s32     %p2, %r8, 256;
        @%p2 bra        LOOP_1;
        mov.f32         %f6, 0f00000000;
        mov.s32         %r14, 0;
        .pragma "nounroll";
LOOP_3:
        mov.f32         %f7, 0f00000000;
        mov.s32         %r15, 0;
        .pragma "nounroll";
LOOP_4:
        shl.b32         %r16, %r6, 6;
        add.s32         %r17, %r16, %r15;
        mad.wide.s32    %rd7, %r17, 4, %rd1;
        ld.global.nc.f32   %f8, [%rd7];
        shl.b32         %r18, %r15, 8;
        add.s32         %r19, %r18, %r14;
        mad.wide.s32    %rd8, %r19, 4, %rd2;
        ld.global.nc.f32   %f9, [%rd8];
        fma.rn.f32      %f7, %f8, %f9, %f7;
        add.s32         %r15, %r15, 1;
        setp.lt.s32     %p3, %r15, 64;
        @%p3 bra        LOOP_4;
        mov.f32         %f10, 0f3E000000;
        mul.f32         %f7, %f7, %f10;
        sub.f32         %f11, %f7, %f1;
        mul.f32         %f13, %f11, 0f3FB8AA3B;
        ex2.approx.ftz.f32 %f12, %f13;
        add.f32         %f6, %f6, %f12;
        add.s32         %r14, %r14, 1;
        setp.lt.s32     %p4, %r14, 256;
        @%p4 bra        LOOP_3;
        rcp.rn.f32      %f14, %f6;
        mov.f32         %f15, 0f00000000;
        mov.s32         %r20, 0;
        .pragma "nounroll";
LOOP_5:
        mov.f32         %f16, 0f00000000;
        mov.s32         %r21, 0;
        .pragma "nounroll";
LOOP_6:
        shl.b32         %r22, %r6, 6;
        add.s32         %r23, %r22, %r21;
        mad.wide.s32    %rd9, %r23, 4, %rd1;
        ld.global.nc.f32   %f17, [%rd9];
        shl.b32         %r24, %r21, 8;
        add.s32         %r25, %r24, %r20;
        mad.wide.s32    %rd10, %r25, 4, %rd2;
        ld.global.nc.f32   %f18, [%rd10];
        fma.rn.f32      %f16, %f17, %f18, %f16;
        add.s32         %r21, %r21, 1;
        setp.lt.s32     %p5, %r21, 64;
        @%p5 bra        LOOP_6;
        mov.f32         %f19, 0f3E000000;
        mul.f32         %f16, %f16, %f19;
        sub.f32         %f20, %f16, %f1;
        mul.f32         %f22, %f20, 0f3FB8AA3B;
        ex2.approx.ftz.f32 %f21, %f22;
        mul.f32         %f23, %f21, %f14;
        shl.b32         %r26, %r20, 6;
        add.s32         %r27, %r26, %r7;
        mad.wide.s32    %rd11, %r27, 4, %rd3;
        ld.global.nc.f32   %f24, [%rd11];
        fma.rn.f32      %f15, %f23, %f24, %f15;
        add.s32         %r20, %r20, 1;
        setp.lt.s32     %p6, %r20, 256;
        @%p6 bra        LOOP_5;
        shl.b32         %r28, %r6, 6;
        add.s32         %r29, %r28, %r7;
        mad.wide.s32    %rd12, %r29, 4, %rd4;
        st.global.f32   [%rd12], %f15;
        ret;
}
