.version 8.0
.target sm_89
.address_size 64

.visible .entry k_select(
        .param .u64 param_x,
        .param .u64 param_out
)
.reqntid 128
{
        .reg .pred      %p<8>;
        .reg .f32       %f<5>;
        .reg .b32       %r<6>;
        .reg .b64       %rd<5>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_out];
        cvta.to.global.u64     %rd2, %rd2;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        mad.wide.s32    %rd3, %r4, 4, %rd1;
        ld.global.nc.f32   %f1, [%rd3];
        mov.f32         %f2, 0f00000000;
        setp.eq.s32     %p1, 0, 1;
        setp.gt.f32    %p2, %f1, %f2;
        not.pred        %p3, %p1;
        and.pred        %p3, %p3, %p2;
        mov.f32         %f4, 0f00000000;
        selp.f32        %f3, %f1, %f4, %p3;
        or.pred         %p4, %p1, %p2;
        setp.ne.s32     %p5, 1, 0;
        not.pred        %p6, %p4;
        and.pred        %p6, %p6, %p5;
        selp.f32        %f3, %f2, %f3, %p6;
        or.pred         %p7, %p4, %p5;
        mad.wide.s32    %rd4, %r4, 4, %rd2;
        st.global.f32   [%rd4], %f3;
        ret;
}
